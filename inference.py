"""Inference entry point: ``python inference.py [group=option] [a.b=value] ...``.

Mirrors the reference's Hydra main (``inference.py:11-20``).
"""

import logging
import sys

import torch.distributed as dist

from neural_scaling_weather_b200 import config as C
from neural_scaling_weather_b200.inference.inferencer import Inferencer


def main(argv=None):
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s")
    name, overrides = C.parse_cli(sys.argv[1:] if argv is None else argv)
    cfg = C.compose(name, overrides)
    inf = Inferencer(cfg)
    out = inf.launch()
    if dist.is_initialized():
        dist.destroy_process_group()
    logging.info("DONE")
    return out


if __name__ == "__main__":
    main()
