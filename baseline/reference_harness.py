"""Drive the unmodified reference code (copied to ``baseline/_ref``) through its own API.

The reference is a plain Python tree without packaging metadata, so ``pip install``
refuses it ("Neither 'setup.py' nor 'pyproject.toml' found"); ``ensure_reference()``
places an unmodified source copy in ``baseline/_ref`` (git-ignored) and it is imported from
there.  The source location comes from the ``NSW_REFERENCE_SRC`` environment variable, or
else from the ``reference_path`` key of ``BASELINE.json`` at the repository root.  The copy
is made by ``__graft_entry__.build()`` and again on demand by ``available()``, so a checkout
that lacks it (a fresh clone, a GPU box that received the tree) fills it when the source is
reachable; the copied tree travels with the repository to machines where it is not.
Packages that its modules import at top level but that are absent on this platform are
replaced by inert stand-ins registered in ``sys.modules`` *before* the import:

* ``omegaconf``: only the ``ListConfig``/``DictConfig`` names are used, for ``isinstance``
  checks and type hints (``models/swin.py:18,62``, ``utils/profiler_utils.py:5``);
* ``matplotlib`` / ``mpl_toolkits``: plotting helpers only;
* ``torch_harmonics``: only the AMSE loss and spectra use it (not on the measured path);
* ``wandb``, ``h5py``, ``nvidia.dali``: logging and the HDF5/DALI readers (not used).

No reference file is modified.  The model, distributed layers, DDP hook, loss, optimizer,
scheduler and the trainer's gradient-norm clipping all run as shipped.
"""

from __future__ import annotations

import json
import os
import shutil
import sys
import types

HERE = os.path.dirname(os.path.abspath(__file__))
REF_ROOT = os.path.join(HERE, "_ref")


class _ListConfig(list):
    pass


class _DictConfig(dict):
    def __getattr__(self, k):
        try:
            return self[k]
        except KeyError:
            raise AttributeError(k) from None

    def __setattr__(self, k, v):
        self[k] = v


def _module(name, **attrs):
    m = types.ModuleType(name)
    m.__dict__.update(attrs)
    return m


def install_stubs():
    if "omegaconf" not in sys.modules:
        oc = _module("omegaconf", ListConfig=_ListConfig, DictConfig=_DictConfig)
        oc.OmegaConf = types.SimpleNamespace(
            to_container=lambda c, **k: dict(c), to_yaml=lambda c: str(c),
            save=lambda *a, **k: None, load=lambda *a, **k: _DictConfig())
        sys.modules["omegaconf"] = oc

    class _Anything(types.ModuleType):
        def __getattr__(self, name):
            if name.startswith("__"):
                raise AttributeError(name)
            return _Anything(f"{self.__name__}.{name}")

        def __call__(self, *a, **k):
            return _Anything(self.__name__ + "()")

    for name in ("matplotlib", "matplotlib.pyplot", "matplotlib.cm", "mpl_toolkits",
                 "mpl_toolkits.axes_grid1", "wandb", "h5py", "nvidia", "nvidia.dali",
                 "nvidia.dali.pipeline", "nvidia.dali.fn", "nvidia.dali.plugin",
                 "nvidia.dali.plugin.pytorch"):
        try:
            __import__(name)
        except Exception:
            sys.modules[name] = _Anything(name)
    try:
        import torch_harmonics  # noqa: F401
    except Exception:
        class RealSHT:  # noqa: D401 - stand-in that fails loudly if used
            def __init__(self, *a, **k):
                raise RuntimeError("torch_harmonics is not installed; AMSE/spectra unavailable")

        sys.modules["torch_harmonics"] = _module("torch_harmonics", RealSHT=RealSHT)


def reference_source() -> str | None:
    """Directory holding the reference's source tree, or None if it is not named anywhere."""
    src = os.environ.get("NSW_REFERENCE_SRC")
    if src:
        return src
    try:
        with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
            return json.load(f).get("reference_path")
    except (OSError, ValueError):
        return None


def _is_tree(path) -> bool:
    return bool(path) and all(os.path.isdir(os.path.join(path, d)) for d in ("models", "distributed", "utils"))


def ensure_reference() -> bool:
    """Copy the reference source tree, unmodified, to ``baseline/_ref`` if it is not there.

    The copy goes to a temporary sibling first and is renamed into place, so a concurrent
    reader never sees a half-written tree.  Returns whether the copy is present afterwards.
    """
    if _is_tree(REF_ROOT):
        return True
    src = reference_source()
    if not _is_tree(src):
        return False
    tmp = f"{REF_ROOT}.tmp{os.getpid()}"
    if os.path.isdir(tmp):
        shutil.rmtree(tmp)
    shutil.copytree(src, tmp, ignore=shutil.ignore_patterns(".git", "__pycache__", "*.pyc"))
    try:
        os.rename(tmp, REF_ROOT)
    except OSError:  # another process placed it first
        shutil.rmtree(tmp, ignore_errors=True)
    return _is_tree(REF_ROOT)


def available() -> bool:
    return ensure_reference()


def import_reference():
    """Return a namespace with the reference modules used by the harness."""
    if not available():
        raise RuntimeError(f"reference source not found under {REF_ROOT}")
    install_stubs()
    if REF_ROOT not in sys.path:
        sys.path.insert(0, REF_ROOT)
    import importlib

    ns = types.SimpleNamespace()
    ns.comm = importlib.import_module("utils.comm")
    ns.helpers = importlib.import_module("distributed.helpers")
    ns.mappings = importlib.import_module("distributed.mappings")
    ns.model_helpers = importlib.import_module("models.helpers")
    ns.swin = importlib.import_module("models.swin")
    ns.swin_helpers = importlib.import_module("models.swin_helpers")
    ns.losses = importlib.import_module("utils.losses")
    ns.optimizer_utils = importlib.import_module("utils.optimizer_utils")
    ns.misc_utils = importlib.import_module("utils.misc_utils")
    ns.flops_utils = importlib.import_module("utils.flops_utils")
    ns.rank_generator = importlib.import_module("utils.rank_generator")
    try:
        ns.trainer = importlib.import_module("utils.trainer")
    except Exception as e:  # pragma: no cover - depends on optional imports
        ns.trainer = None
        ns.trainer_error = e
    return ns


def make_cfg(d):
    """Nested attribute-dict config; lists become the stand-in ListConfig."""
    if isinstance(d, dict):
        return _DictConfig({k: make_cfg(v) for k, v in d.items()})
    if isinstance(d, (list, tuple)):
        return _ListConfig(make_cfg(v) for v in d)
    return d
