"""Training entry point: ``python train.py [group=option] [a.b=value] ...``.

Mirrors the reference's Hydra main (``train.py:10-19``): compose the configuration from
``neural_scaling_weather_b200/config/yaml/default.yaml`` and the command-line
overrides, build the trainer, run it and tear the process group down.
"""

import logging
import sys

import torch.distributed as dist

from neural_scaling_weather_b200 import config as C
from neural_scaling_weather_b200.training.trainer import Trainer


def main(argv=None):
    logging.basicConfig(level=logging.INFO, format="%(asctime)s %(levelname)s %(message)s")
    name, overrides = C.parse_cli(sys.argv[1:] if argv is None else argv)
    cfg = C.compose(name, overrides)
    trainer = Trainer(cfg)
    trainer.launch()
    if dist.is_initialized():
        dist.destroy_process_group()
    logging.info("DONE")
    return trainer


if __name__ == "__main__":
    main()
