"""Generate the golden fixtures of tests/golden/ by running the REFERENCE implementation.

Run in a container where the LightDelta reference sources are present:

    python tests/golden/make_golden.py --reference <path to LightDelta>/python

It imports the reference's own Python code (torch only, on the CPU):
  * lightdelta.reference.post_conv_gdn   (python/lightdelta/reference/gdn.py:70-128)
  * lightdelta.backend.GDNBackend with BackendConfig() -- the Torch-reference + packed-state
    path that the reference's CUDA parity tests use as their expectation
    (tests/test_gdn.py:58-122; python/lightdelta/backend.py:30-91).  The reference module
    ``lightdelta.ops`` only loads the compiled ``_C`` library, which that path never calls, so
    it is replaced by an empty module while the fixtures are made.
Inputs are regenerated from seeds by tests/golden/detrand.py, so a fixture stores only its
case parameters and the reference's results: full bf16 outputs and, for states, values at
seeded sample positions (a few hundred per slot).  Nothing here runs on the GPU box.
"""

from __future__ import annotations

import argparse
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from golden import cases, detrand  # noqa: E402


def _import_reference(path: str):
    sys.path.insert(0, path)
    sys.modules["lightdelta.ops"] = types.ModuleType("lightdelta.ops")
    import lightdelta  # noqa: F401
    from lightdelta.backend import GDNBackend
    from lightdelta.config import BackendConfig
    from lightdelta.reference import GDNInputs, post_conv_gdn

    return GDNBackend, BackendConfig, GDNInputs, post_conv_gdn


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def make_post_conv(post_conv_gdn, GDNInputs) -> None:
    for spec in cases.POST_CONV_CASES:
        arrays = cases.post_conv_inputs(spec)
        dtype = torch.bfloat16 if spec["io_bf16"] else torch.float32

        def tensor(name, cast=True):
            value = torch.from_numpy(arrays[name])
            return value.to(dtype) if cast else value

        inputs = GDNInputs(
            tensor("q"), tensor("k"), tensor("v"), tensor("a"), tensor("b"),
            tensor("a_log", cast=False), tensor("dt_bias", cast=False), tensor("gate"),
            tensor("norm_weight", cast=False),
        )
        result = post_conv_gdn(
            inputs,
            torch.from_numpy(arrays["initial_state"]),
            torch.from_numpy(arrays["lengths"]),
            save_checkpoints=spec["checkpoints"],
            norm_eps=spec["eps"],
        )
        record = {"output": result.output.float().numpy()}
        states = result.checkpoints if spec["checkpoints"] else result.final_state
        states = states.numpy()
        positions = cases.sample_positions(spec["seed"] + 99, states.size, spec["samples"])
        record["state_positions"] = positions
        record["state_values"] = states.reshape(-1)[positions]
        np.savez_compressed(HERE / f"{spec['name']}.npz", **record)
        print(spec["name"], {k: v.shape for k, v in record.items()})


def make_backend(GDNBackend, BackendConfig) -> None:
    for spec in cases.BACKEND_CASES:
        case = cases.backend_case(spec)
        t = {k: torch.from_numpy(v) for k, v in case["arrays"].items()}
        qkvz = t["qkvz_bits"].view(torch.bfloat16)
        ba = t["ba_bits"].view(torch.bfloat16)
        n = case["rows"]
        qkv_width = case["qkv_width"]
        hv = case["hv"]
        kwargs = dict(
            qkv=qkvz[:n, :qkv_width],
            a=ba[:n, hv:],
            b=ba[:n, :hv],
            a_log=t["a_log"],
            dt_bias=t["dt_bias_bits"].view(torch.bfloat16),
            slots=t["slots"],
            cu=t["cu"],
            accepted=t["accepted"],
            pool=t["pool"],
            gate=qkvz[:n, qkv_width:].view(n, hv, 128),
            weight=t["weight_bits"].view(torch.bfloat16),
            out=torch.zeros(n, hv, 128, dtype=torch.bfloat16),
        )
        GDNBackend(BackendConfig())(**kwargs)
        pool = kwargs["pool"].numpy()
        positions = cases.per_slot_positions(spec["seed"] + 77, pool.shape, spec["samples_per_slot"])
        record = {
            "out_bits": _bits(kwargs["out"]),
            "pool_positions": positions,
            "pool_values": pool.reshape(-1)[positions],
        }
        np.savez_compressed(HERE / f"{spec['name']}.npz", **record)
        print(spec["name"], {k: v.shape for k, v in record.items()})


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the reference's python/ directory")
    args = parser.parse_args()
    torch.set_num_threads(8)
    GDNBackend, BackendConfig, GDNInputs, post_conv_gdn = _import_reference(args.reference)
    make_post_conv(post_conv_gdn, GDNInputs)
    make_backend(GDNBackend, BackendConfig)
    return 0


if __name__ == "__main__":
    sys.exit(main())
