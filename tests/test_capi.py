"""CPU tests of the drop-in boundary: the C-ABI library loads and exports every declared
symbol, host-side argument validation, the torch.library schemas match the reference's
(csrc/register.cpp:4-11), and the build loads through the reference's own loader route as
`lightdelta._C`.  Nothing here launches a kernel."""

import ctypes
import re
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "lightdelta_b200.h"

REFERENCE_SCHEMAS = {
    "decode": "lightdelta::decode(Tensor qkv, Tensor a, Tensor b, Tensor a_log, Tensor dt_bias, Tensor indices, "
              "Tensor cu, Tensor accepted, Tensor(s!) state, Tensor gate, Tensor weight, Tensor(o!) out, "
              "float eps) -> ()",
    "gather_state": "lightdelta::gather_state(Tensor pool, Tensor slots, Tensor valid, Tensor(o!) out) -> ()",
    "scatter_state": "lightdelta::scatter_state(Tensor packed, Tensor slots, Tensor(p!) pool) -> ()",
}


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(ld_\w+)\s*\(", text, flags=re.M)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for expected in ("ld_decode", "ld_gather_state", "ld_scatter_state", "ld_copy_slots", "ld_last_error",
                     "ld_version", "ld_fault_flags"):
        assert expected in names


def test_library_exports_every_declared_symbol(native):
    lib = ctypes.CDLL(str(native.LIB_PATH))
    missing = [name for name in declared_functions() if not hasattr(lib, name)]
    assert not missing, f"not exported: {missing}"


def test_version(native):
    assert "sm_100a" in native.version()


def test_decode_rejects_bad_width_before_touching_the_gpu(native):
    rc = native.lib().ld_decode(None, 0, None, 0, None, 0, None, None, 0, None, 4, 5, None, None, None, 1, 0, None, 0,
                                None, 0, None, 0, 16, 32, 1e-6, None)
    assert rc == native.LD_ERR_INVALID
    assert "1 through 4" in native.last_error()


@pytest.mark.parametrize(
    "heads, eps, message",
    [((16, 40), 1e-6, "multiple of num_k_heads"), ((16, 32), 0.0, "epsilon"), ((0, 32), 1e-6, "multiple")],
)
def test_decode_rejects_bad_geometry(native, heads, eps, message):
    rc = native.lib().ld_decode(None, 0, None, 0, None, 0, None, None, 0, None, 4, 1, None, None, None, 1, 0, None, 0,
                                None, 0, None, 0, heads[0], heads[1], eps, None)
    assert rc == native.LD_ERR_INVALID
    assert message in native.last_error()


def test_decode_zero_requests_is_a_no_op(native):
    rc = native.lib().ld_decode(None, 0, None, 0, None, 0, None, None, 0, None, 0, 1, None, None, None, 1, 0, None, 0,
                                None, 0, None, 0, 16, 32, 1e-6, None)
    assert rc == native.LD_OK
    assert native.last_error() == ""


def test_decode_rejects_null_pointers(native):
    rc = native.lib().ld_decode(None, 10240, None, 48, None, 48, None, None, 0, None, 4, 1, None, None, None, 2,
                                786432, None, 6144, None, 0, None, 4, 16, 48, 1e-6, None)
    assert rc == native.LD_ERR_INVALID
    assert "NULL" in native.last_error()


def test_bf16_state_pool_needs_a_slot_stride_divisible_by_8(native):
    """Host-side checks only: the addresses are never dereferenced (the call fails validation)."""
    fake = 1 << 20  # 16-byte aligned, non-NULL
    slot = 48 * 128 * 128
    args = [fake, 10240, fake, 48, fake, 48, fake, fake, 0, fake, 4, 1, fake, fake, fake, 2, slot + 4, fake, 6144,
            fake, 0, fake, 4, 16, 48, 1e-6, None]
    assert native.lib().ld_decode_bf16_state(*args) == native.LD_ERR_INVALID
    assert "divisible by 8" in native.last_error()


def test_state_io_validation(native):
    lib = native.lib()
    assert lib.ld_gather_state(None, 4, 16, None, 1, None, 0, None, 16, 16, None) == native.LD_OK
    assert lib.ld_gather_state(None, 4, 16, None, 1, None, 3, None, 16, 16, None) == native.LD_ERR_INVALID
    assert lib.ld_scatter_state(None, 16, None, 1, 2, None, 4, 8, 16, None) == native.LD_ERR_INVALID
    assert "NULL" in native.last_error() or "stride" in native.last_error()
    assert lib.ld_copy_slots(None, 0, 16, None, 1, None, 1, 2, 16, None) == native.LD_ERR_INVALID
    assert "at least one slot" in native.last_error()


def test_torch_schemas_match_the_reference(native):
    from lightdelta_b200 import ops  # noqa: F401

    for name, schema in REFERENCE_SCHEMAS.items():
        assert str(getattr(torch.ops.lightdelta, name).default._schema) == schema


def test_fake_kernels_allow_tracing(native):
    from torch._subclasses.fake_tensor import FakeTensorMode

    from lightdelta_b200 import ops  # noqa: F401

    with FakeTensorMode():
        pool = torch.empty(4, 2, 128, 128)
        slots = torch.zeros(3, dtype=torch.int32)
        valid = torch.zeros(3, dtype=torch.bool)
        packed = torch.empty(3, 2, 128, 128)
        assert torch.ops.lightdelta.gather_state(pool, slots, valid, packed) is None
        assert torch.ops.lightdelta.scatter_state(packed, slots, pool) is None


def test_cpu_tensors_have_no_kernel(native):
    """The ops are registered for CUDA only: CPU tensors fail loudly instead of falling back."""
    from lightdelta_b200 import ops  # noqa: F401

    pool = torch.zeros(2, 1, 4, 4)
    with pytest.raises((RuntimeError, NotImplementedError)):
        torch.ops.lightdelta.scatter_state(torch.zeros(1, 1, 4, 4), torch.ones(1, dtype=torch.int32), pool)


def test_process_wide_toggles(native):
    """Kernel override and programmatic-launch switches: set, query and restore (no launch)."""
    lib = native.lib()
    previous = lib.ld_decode_kernel_override(native.DECODE_KERNELS["rowreg"])
    assert lib.ld_decode_kernel_override(previous) == native.DECODE_KERNELS["rowreg"]
    assert lib.ld_decode_kernel_override(99) == -native.LD_ERR_INVALID
    enabled = lib.ld_programmatic_launch(-1)
    assert enabled in (0, 1)
    assert lib.ld_programmatic_launch(0) == enabled
    assert lib.ld_programmatic_launch(-1) == 0
    assert lib.ld_programmatic_launch(enabled) == 0
    assert lib.ld_programmatic_launch(-1) == enabled


def test_wait_test_hook_checks_its_arguments(native):
    lib = native.lib()
    assert lib.ld_decode_wait_test(-1, 0) == native.LD_ERR_INVALID
    assert lib.ld_decode_wait_test(0, 4096) == native.LD_ERR_INVALID
    assert lib.ld_decode_wait_test(0, 0) == native.LD_OK


def test_loads_as_the_reference_package_extension(native, tmp_path):
    """The drop-in route of the reference's loader (python/lightdelta/ops/__init__.py:7 finds
    `lightdelta._C` with importlib and loads it with torch.ops.load_library): with the two
    libraries installed as that package's `_C.so`, the reference's three schemas register."""
    import json
    import shutil
    import subprocess
    import sys

    package = tmp_path / "lightdelta"
    package.mkdir()
    (package / "__init__.py").write_text("")
    shutil.copy(native.LIB_PATH.parent / "_C.so", package / "_C.so")
    shutil.copy(native.LIB_PATH, package / native.LIB_PATH.name)
    script = (
        "import importlib.util, json, torch\n"
        "torch.ops.load_library(importlib.util.find_spec('lightdelta._C').origin)\n"
        "print(json.dumps({n: str(getattr(torch.ops.lightdelta, n).default._schema)"
        " for n in ('decode', 'gather_state', 'scatter_state')}))\n"
    )
    result = subprocess.run([sys.executable, "-c", script], cwd=tmp_path, capture_output=True, text=True,
                            timeout=300, check=True)
    assert json.loads(result.stdout.strip().splitlines()[-1]) == REFERENCE_SCHEMAS
