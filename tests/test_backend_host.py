"""CPU tests of the host side of the backend boundary: BackendConfig (the rules of
python/lightdelta/config.py:7-60, restated) and GDNBackend's checks made before any launch."""

import pytest
import torch

from lightdelta_b200.config import BackendConfig


def write(tmp_path, text):
    path = tmp_path / "config.toml"
    path.write_text(text)
    return path


def test_defaults_are_valid():
    BackendConfig().validate()


def test_a_full_config_loads(tmp_path):
    path = write(tmp_path, """
[gdn]
compute = "cuda_fused"
state_io = "indexed"
prefill_io = "fused_copy"

[runtime]
cuda_graph = true

[speculation]
method = "mtp"
num_speculative_tokens = 3
""")
    config = BackendConfig.from_file(path)
    assert (config.compute, config.state_io, config.prefill_io, config.cuda_graph) == (
        "cuda_fused", "indexed", "fused_copy", True)
    assert (config.speculation_method, config.num_speculative_tokens) == ("mtp", 3)


@pytest.mark.parametrize("text, message", [
    ("[model]\nx = 1\n", "Unknown config sections"),
    ("[gdn]\nbackend = \"x\"\n", "Unknown keys"),
    ("[gdn]\ncompute = 1\n", "Invalid type"),
    ("[gdn]\ncompute = \"triton\"\n", "compute must be"),
    ("[gdn]\nstate_io = \"paged\"\n", "state_io must be"),
    ("[gdn]\nprefill_io = \"x\"\n", "prefill_io must be"),
    ("[runtime]\ntorch_compile = true\n", "torch.compile is disabled"),
    ("[gdn]\nstate_io = \"indexed\"\n", "Torch reference requires"),
    ("[speculation]\nnum_speculative_tokens = 2\n", "none speculation"),
    ("[gdn]\ncompute = \"cuda_fused\"\n[speculation]\nmethod = \"mtp\"\nnum_speculative_tokens = 4\n", "MTP requires"),
])
def test_invalid_configs_raise(tmp_path, text, message):
    with pytest.raises(ValueError, match=message):
        BackendConfig.from_file(write(tmp_path, text))


def test_backend_offers_only_the_fused_compute(native):
    from lightdelta_b200.backend import GDNBackend

    with pytest.raises(ValueError, match="cuda_fused"):
        GDNBackend(BackendConfig())


def test_packed_mode_refuses_a_bf16_pool_before_launching(native):
    from lightdelta_b200.backend import GDNBackend

    backend = GDNBackend(BackendConfig(compute="cuda_fused", state_io="packed"))
    slots = torch.ones(2, 1, dtype=torch.int32)
    pool = torch.zeros(3, 2, 128, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="fp32 pool"):
        backend(None, None, None, None, None, slots, None, None, pool, None, None, None)


def test_the_reference_config_files_load_unchanged():
    """Every configs/*.toml of the reference checkout (when it sits beside this repository) loads,
    and each field agrees with a plain TOML read of the file."""
    import tomllib
    from pathlib import Path

    configs = Path(__file__).resolve().parent.parent.parent / "reference" / "configs"
    files = sorted(configs.glob("*.toml")) if configs.is_dir() else []
    if not files:
        pytest.skip("reference checkout not present")
    for path in files:
        config = BackendConfig.from_file(path)
        raw = tomllib.loads(path.read_text())
        for section, attr_of in (("gdn", {}), ("runtime", {}),
                                 ("speculation", {"method": "speculation_method"})):
            for key, value in raw.get(section, {}).items():
                assert getattr(config, attr_of.get(key, key)) == value, (path.name, key)


def test_schema_covers_every_field_and_default():
    from lightdelta_b200 import config as cfg

    assert [o.attr for o in cfg.SCHEMA] == list(BackendConfig.__dataclass_fields__)
    defaults = BackendConfig()
    assert all(getattr(defaults, o.attr) == o.default for o in cfg.SCHEMA)


def test_bool_is_not_accepted_for_an_int_field():
    with pytest.raises(ValueError, match="Invalid type for num_speculative_tokens"):
        BackendConfig(speculation_method="mtp", num_speculative_tokens=True).validate()


def test_backend_accepts_the_callers_own_config_object(native):
    """The reference's callers build its own BackendConfig; GDNBackend reads compute and
    state_io from any such object after calling its validate()."""
    from types import SimpleNamespace

    from lightdelta_b200.backend import GDNBackend

    calls = []
    foreign = SimpleNamespace(compute="cuda_fused", state_io="indexed", validate=lambda: calls.append(1))
    backend = GDNBackend(foreign)
    assert backend.config is foreign and calls == [1]
    with pytest.raises(ValueError, match="state_io must be"):
        GDNBackend(SimpleNamespace(compute="cuda_fused", state_io="paged", validate=lambda: None))
