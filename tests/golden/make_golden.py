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
  * LightDeltaRejectionSampler (python/lightdelta/runtime/speculation.py:271-326), loaded from
    its file with the vLLM modules it imports at the top replaced by empty stand-ins: the
    sampler itself uses torch only.
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


class _Stub(types.ModuleType):
    """Module whose every attribute is a placeholder class (import-time names only)."""

    def __getattr__(self, name):
        if name.startswith("__"):
            raise AttributeError(name)
        return type(name, (), {})


class _SamplerOutput:
    FIELDS = ("sampled_token_ids", "logprobs_tensors", "num_nans", "num_sampled", "num_rejected")

    def __init__(self, *values):
        for field, value in zip(self.FIELDS, values):
            setattr(self, field, value)


def _import_sampler(path: str):
    import importlib.util

    names = ["vllm", "vllm.config", "vllm.config.compilation", "vllm.forward_context", "vllm.model_executor",
             "vllm.model_executor.layers", "vllm.model_executor.layers.attention_layer_base", "vllm.v1",
             "vllm.v1.worker", "vllm.v1.worker.gpu", "vllm.v1.worker.gpu.attn_utils",
             "vllm.v1.worker.gpu.input_batch", "vllm.v1.worker.gpu.sample", "vllm.v1.worker.gpu.sample.output",
             "vllm.v1.worker.gpu.spec_decode", "vllm.v1.worker.gpu.spec_decode.eagle",
             "vllm.v1.worker.gpu.spec_decode.eagle.utils"]
    saved = {name: sys.modules.get(name) for name in names}
    for name in names:
        sys.modules[name] = _Stub(name)
    sys.modules["vllm.v1.worker.gpu.sample.output"].SamplerOutput = _SamplerOutput
    try:
        file = Path(path) / "lightdelta" / "runtime" / "speculation.py"
        spec = importlib.util.spec_from_file_location("reference_speculation", file)
        module = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(module)
    finally:
        for name, module_before in saved.items():
            if module_before is None:
                sys.modules.pop(name, None)
            else:
                sys.modules[name] = module_before
    return module.LightDeltaRejectionSampler


def make_sampler(LightDeltaRejectionSampler) -> None:
    from types import SimpleNamespace

    dtypes = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}
    for spec in cases.SAMPLER_CASES:
        case = cases.sampler_case(spec)
        token_dtype = torch.int64 if spec["tokens"] == "i64" else torch.int32
        batch = SimpleNamespace(
            num_reqs=spec["requests"],
            num_draft_tokens_per_req=case["num_draft_tokens"].copy(),
            input_ids=torch.from_numpy(case["input_ids"]).to(token_dtype),
            query_start_loc=torch.from_numpy(case["query_start_loc"]),
            cu_num_logits=torch.from_numpy(case["cu_num_logits"]),
            seq_lens=torch.from_numpy(case["seq_lens"]),
            prefill_len_np=case["prefill_len"].copy(),
        )
        logits = torch.from_numpy(case["logits"]).to(dtypes[spec["dtype"]])
        output = LightDeltaRejectionSampler(spec["steps"])(logits, batch)
        record = {
            "target": logits.argmax(dim=-1).numpy(),  # speculation.py:279
            "sampled": output.sampled_token_ids.to(torch.int64).numpy(),
            "num_sampled": output.num_sampled.numpy(),
            "num_rejected": output.num_rejected.numpy(),
        }
        np.savez_compressed(HERE / f"{spec['name']}.npz", **record)
        print(spec["name"], {k: v.shape for k, v in record.items()})


def main() -> int:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", required=True, help="path of the reference's python/ directory")
    parser.add_argument("--only", choices=("all", "gdn", "sampler"), default="all")
    args = parser.parse_args()
    torch.set_num_threads(8)
    if args.only in ("all", "gdn"):
        GDNBackend, BackendConfig, GDNInputs, post_conv_gdn = _import_reference(args.reference)
        make_post_conv(post_conv_gdn, GDNInputs)
        make_backend(GDNBackend, BackendConfig)
    if args.only in ("all", "sampler"):
        make_sampler(_import_sampler(args.reference))
    return 0


if __name__ == "__main__":
    sys.exit(main())
