"""Hierarchical YAML configuration with a Hydra-compatible command-line surface.

The reference composes its configuration with Hydra 1.x
(``train.py:10`` ``@hydra.main(config_path="config", config_name="default")``) from the
tree under ``config/`` (``config/default.yaml:1-18``).  Hydra and omegaconf are not
available on this platform, so this module implements the subset of that behaviour the
framework's entry points use:

* a defaults list (``group: option``, ``_self_``, ``group: null``) resolved against the
  YAML files under ``config/yaml/<group>/<option>.yaml``;
* ``# @package _global_`` overlays (the ``debug`` group) merged at the root;
* command-line overrides ``group=option``, ``a.b=value``, ``+a.b=value`` (add) and
  ``~a.b`` (delete), values parsed as YAML scalars/lists;
* ``${a.b}`` interpolation, resolved on access and by :func:`to_container`;
* saving the resolved config as ``hyperparameters.yaml`` and loading it back.

:class:`Config` is a ``dict`` with attribute access, so ``cfg.model.embed_dim`` and
``getattr(cfg.model, "coord_pos_embed", True)`` behave as they do on an omegaconf
``DictConfig``.
"""

from __future__ import annotations

import copy
import os
import re
from typing import Any, Iterable, List, Optional

import yaml

CONFIG_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "yaml")

_INTERP = re.compile(r"\$\{([^}]+)\}")


class _Loader(yaml.SafeLoader):
    """SafeLoader that also reads ``5E-4``/``1e-4`` (no dot) as floats, as omegaconf does."""


_Loader.add_implicit_resolver(
    "tag:yaml.org,2002:float",
    re.compile(r"""^(?:[-+]?(?:[0-9][0-9_]*)\.[0-9_]*(?:[eE][-+]?[0-9]+)?
    |[-+]?(?:[0-9][0-9_]*)(?:[eE][-+]?[0-9]+)
    |\.[0-9_]+(?:[eE][-+][0-9]+)?
    |[-+]?\.(?:inf|Inf|INF)
    |\.(?:nan|NaN|NAN))$""", re.X),
    list("-+0123456789."))


def _yaml_load(text):
    return yaml.load(text, Loader=_Loader)


class ConfigError(KeyError):
    pass


class Config(dict):
    """A nested dict with attribute access and lazy ``${...}`` interpolation."""

    def __init__(self, *args, _root: Optional["Config"] = None, **kwargs):
        super().__init__()
        object.__setattr__(self, "_root", _root)
        data = dict(*args, **kwargs)
        for k, v in data.items():
            self[k] = v

    # -- structure ---------------------------------------------------------
    def _wrap(self, value):
        root = self._root if self._root is not None else self
        if isinstance(value, Config):
            value = dict(value)
        if isinstance(value, dict):
            c = Config(_root=root)
            for k, v in value.items():
                c[k] = v
            return c
        if isinstance(value, (list, tuple)):
            return ListConfig(self._wrap(v) for v in value)
        return value

    def __setitem__(self, key, value):
        super().__setitem__(key, self._wrap(value))

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        try:
            return self[name]
        except KeyError:
            raise AttributeError(name) from None

    def __setattr__(self, name, value):
        self[name] = value

    def __delattr__(self, name):
        try:
            del self[name]
        except KeyError:
            raise AttributeError(name) from None

    def __getitem__(self, key):
        value = super().__getitem__(key)
        return self._resolve(value)

    def get(self, key, default=None):
        if key in self:
            return self[key]
        return default

    def items(self):
        return [(k, self[k]) for k in self.keys()]

    def values(self):
        return [self[k] for k in self.keys()]

    def raw(self, key):
        return super().__getitem__(key)

    def __deepcopy__(self, memo):
        return Config(to_container(self, resolve=False))

    def copy(self):
        return copy.deepcopy(self)

    # -- interpolation -----------------------------------------------------
    def _resolve(self, value):
        if isinstance(value, str) and "${" in value:
            root = self._root if self._root is not None else self
            return _interpolate(root, value)
        return value

    def select(self, dotted: str, default=None):
        node: Any = self
        for part in dotted.split("."):
            if isinstance(node, dict) and part in node:
                node = node[part]
            else:
                return default
        return node


class ListConfig(list):
    """List node of a :class:`Config` (a plain list subclass)."""


def _interpolate(root: Config, text: str, _depth: int = 0):
    if _depth > 32:
        raise ConfigError(f"interpolation depth exceeded for {text!r}")
    whole = _INTERP.fullmatch(text)
    if whole:
        value = root.select(whole.group(1).strip(), default=_MISSING)
        if value is _MISSING:
            raise ConfigError(f"cannot resolve interpolation {text!r}")
        if isinstance(value, str) and "${" in value:
            return _interpolate(root, value, _depth + 1)
        return value

    def repl(m):
        value = root.select(m.group(1).strip(), default=_MISSING)
        if value is _MISSING:
            raise ConfigError(f"cannot resolve interpolation {m.group(0)!r}")
        if isinstance(value, str) and "${" in value:
            value = _interpolate(root, value, _depth + 1)
        return str(value)

    return _INTERP.sub(repl, text)


class _Missing:
    pass


_MISSING = _Missing()


# ---------------------------------------------------------------------------
# conversion helpers


def to_container(cfg, resolve: bool = True):
    """Plain ``dict``/``list`` copy of a config (interpolations resolved if asked)."""
    if isinstance(cfg, Config):
        out = {}
        for k in cfg.keys():
            v = cfg[k] if resolve else cfg.raw(k)
            out[k] = to_container(v, resolve)
        return out
    if isinstance(cfg, (list, tuple)):
        return [to_container(v, resolve) for v in cfg]
    return cfg


def to_yaml(cfg, resolve: bool = False) -> str:
    return yaml.safe_dump(to_container(cfg, resolve=resolve), sort_keys=False)


def save(cfg, path: str, resolve: bool = False) -> None:
    with open(path, "w") as f:
        f.write(to_yaml(cfg, resolve=resolve))


def load(path: str) -> Config:
    with open(path) as f:
        data = _yaml_load(f) or {}
    return Config(data)


def create(data: dict) -> Config:
    return Config(copy.deepcopy(data))


# ---------------------------------------------------------------------------
# composition


def _read_yaml(path: str):
    with open(path) as f:
        text = f.read()
    package_global = any(
        line.strip().replace(" ", "") == "#@package_global_" for line in text.splitlines()[:5]
    )
    data = _yaml_load(text) or {}
    return data, package_global


def _deep_merge(dst: dict, src: dict) -> dict:
    for k, v in src.items():
        if isinstance(v, dict) and isinstance(dst.get(k), dict):
            _deep_merge(dst[k], v)
        else:
            dst[k] = copy.deepcopy(v)
    return dst


def _parse_value(text: str):
    if text == "":
        return ""
    try:
        return _yaml_load(text)
    except yaml.YAMLError:
        return text


def _split_overrides(overrides: Iterable[str], groups: List[str]):
    group_choice = {}
    value_ovr = []
    for ov in overrides:
        ov = ov.strip()
        if not ov:
            continue
        if ov.startswith("~"):
            value_ovr.append(("del", ov[1:].split("=")[0], None))
            continue
        if "=" not in ov:
            raise ConfigError(f"override {ov!r} is not of the form key=value")
        key, val = ov.split("=", 1)
        add = key.startswith("+")
        key = key.lstrip("+")
        if key in groups and "." not in key:
            group_choice[key] = None if val in ("null", "None", "") else val
        else:
            value_ovr.append(("add" if add else "set", key, _parse_value(val)))
    return group_choice, value_ovr


def _set_dotted(data: dict, dotted: str, value, must_exist: bool):
    parts = dotted.split(".")
    node = data
    for p in parts[:-1]:
        if p not in node or not isinstance(node[p], dict):
            if must_exist:
                raise ConfigError(f"override key {dotted!r} not found in config")
            node[p] = {}
        node = node[p]
    if must_exist and parts[-1] not in node:
        raise ConfigError(
            f"override key {dotted!r} not found in config (use +{dotted}=... to add it)"
        )
    node[parts[-1]] = value


def _del_dotted(data: dict, dotted: str):
    parts = dotted.split(".")
    node = data
    for p in parts[:-1]:
        node = node[p]
    del node[parts[-1]]


def compose(
    config_name: str = "default",
    overrides: Optional[Iterable[str]] = None,
    config_dir: str = CONFIG_DIR,
) -> Config:
    """Compose ``<config_dir>/<config_name>.yaml`` with its defaults list and overrides."""
    overrides = list(overrides or [])
    primary, _ = _read_yaml(os.path.join(config_dir, config_name + ".yaml"))
    defaults = primary.pop("defaults", [])
    groups = []
    for entry in defaults:
        if isinstance(entry, dict):
            groups.extend(entry.keys())
    group_choice, value_ovr = _split_overrides(overrides, groups)

    out: dict = {}
    for entry in defaults:
        if entry == "_self_":
            _deep_merge(out, primary)
            continue
        if isinstance(entry, str):
            data, _ = _read_yaml(os.path.join(config_dir, entry + ".yaml"))
            _deep_merge(out, data)
            continue
        for group, option in entry.items():
            option = group_choice.get(group, option)
            if option is None:
                continue
            path = os.path.join(config_dir, group, f"{option}.yaml")
            if not os.path.isfile(path):
                raise ConfigError(f"no config option {group}={option} ({path})")
            data, is_global = _read_yaml(path)
            if is_global:
                _deep_merge(out, data)
            else:
                out.setdefault(group, {})
                if isinstance(out[group], dict):
                    _deep_merge(out[group], data)
                else:
                    out[group] = data
    if "_self_" not in defaults:
        _deep_merge(out, primary)

    for kind, key, val in value_ovr:
        if kind == "del":
            _del_dotted(out, key)
        else:
            _set_dotted(out, key, val, must_exist=(kind == "set"))
    return Config(out)


def parse_cli(argv: List[str]):
    """Split ``argv`` into (config_name, overrides); ``--config-name X`` is honoured."""
    name = "default"
    ovr = []
    it = iter(argv)
    for a in it:
        if a in ("--config-name", "-cn"):
            name = next(it)
        elif a.startswith("--config-name="):
            name = a.split("=", 1)[1]
        else:
            ovr.append(a)
    return name, ovr


__all__ = [
    "Config",
    "ListConfig",
    "ConfigError",
    "compose",
    "create",
    "load",
    "save",
    "to_container",
    "to_yaml",
    "parse_cli",
    "CONFIG_DIR",
]
