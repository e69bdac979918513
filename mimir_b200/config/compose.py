"""A small Hydra-compatible configuration composer.

The reference composes ``mimir.conf/train.yaml`` with Hydra 1.3
(``src/mimir/training/entry.py:5-10``) and passes CLI overrides through unchanged
(``src/mimir/cli.py:11-15``).  Hydra is not a dependency of this framework, so this
module implements the subset of Hydra's override grammar that the Mimir configuration
tree uses:

* a ``defaults`` list with ``group@package: option`` entries and ``_self_``;
* ``group@package=option`` and ``group=option`` overrides that swap a default;
* ``+group=option`` for optional groups (``+experiment=looped``) whose files may carry
  ``# @package _global_``;
* dotted ``a.b=c`` overrides of existing keys, ``+a.b=c`` to add a key, ``++a.b=c`` to
  add or override, and ``~a.b`` to delete;
* YAML-typed values (``[1,2]``, ``null``, ``true``, numbers, ``{a: 1}``).

Values that are still ``???`` after composition raise ``MissingValueError`` when the
result is validated, like Hydra's mandatory-value check.
"""
from __future__ import annotations

import copy
import os
from pathlib import Path
from typing import Any, Iterable

import yaml

CONF_ROOT = Path(__file__).resolve().parent.parent / "conf"
MISSING = "???"


class ComposeError(ValueError):
    pass


class MissingValueError(ComposeError):
    pass


def _load_yaml(path: Path) -> tuple[dict, str | None]:
    text = path.read_text()
    package = None
    for line in text.splitlines():
        stripped = line.strip()
        if stripped.startswith("# @package"):
            package = stripped.split(None, 2)[2].strip()
            break
        if stripped and not stripped.startswith("#"):
            break
    data = yaml.safe_load(text) or {}
    if not isinstance(data, dict):
        raise ComposeError(f"{path} must contain a mapping")
    return data, package


def _merge(dst: dict, src: dict) -> dict:
    for key, value in src.items():
        if isinstance(value, dict) and isinstance(dst.get(key), dict):
            _merge(dst[key], value)
        else:
            dst[key] = copy.deepcopy(value)
    return dst


def _place(root: dict, package: str | None, data: dict) -> None:
    if package in (None, "", "_global_"):
        _merge(root, data)
        return
    node = root
    for part in package.split("."):
        node = node.setdefault(part, {})
    _merge(node, data)


def _parse_value(text: str) -> Any:
    if text == "":
        return ""
    try:
        return yaml.safe_load(text)
    except yaml.YAMLError:
        return text


def _split_override(item: str) -> tuple[str, str, str | None]:
    """Return (prefix, key, value) where prefix is '', '+', '++' or '~'."""
    prefix = ""
    for candidate in ("++", "+", "~"):
        if item.startswith(candidate):
            prefix, item = candidate, item[len(candidate):]
            break
    if "=" not in item:
        if prefix == "~":
            return prefix, item, None
        raise ComposeError(f"Override '{item}' is missing '='")
    key, value = item.split("=", 1)
    return prefix, key.strip(), value


class Composer:
    """Compose a named root config with overrides."""

    def __init__(self, root: Path | str = CONF_ROOT):
        self.root = Path(root)

    def groups(self) -> set[str]:
        return {p.name for p in self.root.iterdir() if p.is_dir()}

    def options(self, group: str) -> list[str]:
        return sorted(p.stem for p in (self.root / group).glob("*.yaml"))

    def _group_file(self, group: str, option: str) -> Path:
        path = self.root / group / f"{option}.yaml"
        if not path.exists():
            raise ComposeError(
                f"Could not find '{group}/{option}'. Available options in '{group}': {self.options(group)}")
        return path

    def compose(self, config_name: str = "train", overrides: Iterable[str] = ()) -> dict:
        overrides = list(overrides)
        root_data, _ = _load_yaml(self.root / f"{config_name}.yaml")
        defaults = root_data.pop("defaults", [])
        # Resolve the defaults list: (group, package) -> option, in declared order.
        entries: list[tuple[str, str | None, str | None]] = []  # (group, package, option); group '_self_'
        for entry in defaults:
            if entry == "_self_":
                entries.append(("_self_", None, None))
                continue
            if not isinstance(entry, dict) or len(entry) != 1:
                raise ComposeError(f"Bad defaults entry {entry!r}")
            (spec, option), = entry.items()
            group, _, package = spec.partition("@")
            entries.append((group, package or None, option))

        value_overrides: list[tuple[str, str, str | None]] = []
        for item in overrides:
            prefix, key, value = _split_override(item)
            group, _, package = key.partition("@")
            if prefix != "~" and group in self.groups() and "." not in group:
                matched = False
                for index, (g, p, _o) in enumerate(entries):
                    if g == group and (not package or p == package):
                        entries[index] = (g, p, value)
                        matched = True
                if not matched:
                    if prefix not in ("+", "++"):
                        raise ComposeError(
                            f"Could not override '{key}'. To append to your default list use +{key}={value}")
                    entries.append((group, package or None, value))
                continue
            value_overrides.append((prefix, key, value))

        result: dict = {}
        for group, package, option in entries:
            if group == "_self_":
                _merge(result, root_data)
                continue
            if option is None:
                continue
            data, file_package = _load_yaml(self._group_file(group, str(option)))
            target = package if package is not None else (file_package if file_package is not None else group)
            _place(result, target, data)

        for prefix, key, value in value_overrides:
            self._apply(result, prefix, key, value)
        return result

    @staticmethod
    def _apply(cfg: dict, prefix: str, key: str, value: str | None) -> None:
        parts = key.split(".")
        node = cfg
        for part in parts[:-1]:
            if part not in node:
                if prefix in ("+", "++"):
                    node[part] = {}
                else:
                    raise ComposeError(f"Key '{key}' is not in struct")
            node = node[part]
            if not isinstance(node, dict):
                raise ComposeError(f"Key '{key}' traverses a non-mapping")
        leaf = parts[-1]
        if prefix == "~":
            if leaf not in node:
                raise ComposeError(f"Could not delete '{key}': not found")
            del node[leaf]
            return
        exists = leaf in node
        if prefix == "" and not exists:
            raise ComposeError(
                f"Could not override '{key}'. Key '{key}' is not in struct. To append use +{key}={value}")
        if prefix == "+" and exists:
            raise ComposeError(f"Could not append to config. An item is already at '{key}'")
        node[leaf] = _parse_value(value)


def find_missing(cfg: Any, path: str = "") -> list[str]:
    missing = []
    if isinstance(cfg, dict):
        for key, value in cfg.items():
            missing.extend(find_missing(value, f"{path}.{key}" if path else str(key)))
    elif cfg == MISSING:
        missing.append(path)
    return missing


def compose(overrides: Iterable[str] = (), config_name: str = "train",
            root: Path | str | None = None) -> dict:
    root = root or os.environ.get("MIMIR_CONF_ROOT") or CONF_ROOT
    return Composer(root).compose(config_name, overrides)
