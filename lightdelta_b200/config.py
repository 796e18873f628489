"""Backend configuration: the reference's TOML format (python/lightdelta/config.py), read and
checked by a declarative table.

The reference's ``configs/*.toml`` files and its ``BackendConfig`` objects are the interface:
their sections, keys, defaults, allowed values and error messages are kept, so its config files
load unchanged and its callers see the same errors.  The checking here is table driven: ``SCHEMA``
lists every option once (TOML location, attribute, default, allowed values) and ``RULES`` the
rules that relate options to each other.

``GDNBackend`` needs only ``compute`` and ``state_io`` and reads them from any object that has
them, so the reference's own ``BackendConfig`` instances work as well as this one.
"""

from __future__ import annotations

import tomllib
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Callable, NamedTuple


class Option(NamedTuple):
    section: str           # TOML table
    key: str               # key inside the table
    attr: str              # BackendConfig attribute
    default: Any
    allowed: tuple | None  # permitted values (None: any value of the default's type)
    message: str = ""      # error for a value outside `allowed` (default: "<attr> must be a or b")


SCHEMA: tuple[Option, ...] = (
    Option("gdn", "compute", "compute", "torch_reference", ("torch_reference", "cuda_fused")),
    Option("gdn", "state_io", "state_io", "packed", ("packed", "indexed")),
    Option("gdn", "prefill_io", "prefill_io", "reference", ("reference", "fused_copy")),
    Option("runtime", "torch_compile", "torch_compile", False, (False,),
           "torch.compile is disabled for controlled ablations"),
    Option("runtime", "cuda_graph", "cuda_graph", False, None),
    Option("speculation", "method", "speculation_method", "none", None),
    Option("speculation", "num_speculative_tokens", "num_speculative_tokens", 0, None),
)


def _torch_compute_is_eager(c) -> bool:
    return c.compute != "torch_reference" or (c.state_io == "packed" and not c.cuda_graph)


def _no_drafts_without_speculation(c) -> bool:
    return c.speculation_method != "none" or c.num_speculative_tokens == 0


def _mtp_draft_count(c) -> bool:
    return c.speculation_method == "none" or (c.speculation_method == "mtp" and c.num_speculative_tokens in (1, 2, 3))


RULES: tuple[tuple[Callable[[Any], bool], str], ...] = (
    (_torch_compute_is_eager, "Torch reference requires packed state and eager execution"),
    (_no_drafts_without_speculation, "none speculation requires zero draft tokens"),
    (_mtp_draft_count, "MTP requires 1, 2 or 3 draft tokens"),
)


def check(config) -> None:
    """Raises ValueError with the reference's message for the first broken option or rule."""
    for option in SCHEMA:
        value = getattr(config, option.attr)
        if type(value) is not type(option.default):
            raise ValueError(f"Invalid type for {option.attr}")
    for option in SCHEMA:
        value = getattr(config, option.attr)
        if option.allowed is not None and value not in option.allowed:
            raise ValueError(option.message or f"{option.attr} must be {' or '.join(option.allowed)}")
    for holds, message in RULES:
        if not holds(config):
            raise ValueError(message)


@dataclass(frozen=True)
class BackendConfig:
    compute: str = "torch_reference"
    state_io: str = "packed"
    prefill_io: str = "reference"
    torch_compile: bool = False
    cuda_graph: bool = False
    speculation_method: str = "none"
    num_speculative_tokens: int = 0

    def validate(self) -> None:
        check(self)

    @classmethod
    def from_file(cls, path: str | Path) -> "BackendConfig":
        tables = tomllib.loads(Path(path).read_text())
        keys_of: dict[str, set[str]] = {}
        for option in SCHEMA:
            keys_of.setdefault(option.section, set()).add(option.key)
        stray = set(tables) - set(keys_of)
        if stray:
            raise ValueError(f"Unknown config sections: {stray}")
        for section, table in tables.items():
            if not isinstance(table, dict) or set(table) - keys_of[section]:
                raise ValueError(f"Unknown keys or invalid table in [{section}]")
        values = {option.attr: tables.get(option.section, {}).get(option.key, option.default) for option in SCHEMA}
        config = cls(**values)
        config.validate()
        return config


assert tuple(BackendConfig.__dataclass_fields__) == tuple(o.attr for o in SCHEMA), "SCHEMA lists every field"
assert all(BackendConfig.__dataclass_fields__[o.attr].default == o.default for o in SCHEMA)
