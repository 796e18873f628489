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
