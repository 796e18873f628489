"""Generate the conv-update golden fixtures of tests/golden/ by running vLLM's own kernel.

    python tests/golden/make_golden_conv.py

The algorithm is vLLM's causal_conv1d_update (vllm/model_executor/layers/mamba/ops/
causal_conv1d.py), which the reference calls at python/lightdelta/integration/vllm_layer.py:
161-172 and :199-207.  The reference pins vLLM 0.29.0; the image has vLLM 0.22, whose
speculative-decode path takes the same arguments.  Its Triton kernel runs here on the CPU
under Triton's interpreter (TRITON_INTERPRET=1), in fp32 (the interpreter's bf16 emulation
is not exact), which pins the index semantics: window offset accepted - 1, the one-position
shift of the speculative path, the null conv slot, zero-length requests and both state layouts.
Inputs are regenerated from seeds (tests/golden/detrand.py); a fixture holds the outputs and
the new state of every request's slot.  Nothing here runs on the GPU box.
"""

from __future__ import annotations

import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))
from golden import cases  # noqa: E402


def main() -> int:
    from vllm.model_executor.layers.mamba.ops.causal_conv1d import causal_conv1d_update

    for spec in cases.CONV_CASES:
        case = cases.conv_case(spec)
        state = torch.from_numpy(case["state"].copy())
        view = state if spec["layout"] == "dim_first" else state.transpose(1, 2)
        x = torch.from_numpy(case["x"].copy())
        weight = torch.from_numpy(case["weight"])
        bias = None if case["bias"] is None else torch.from_numpy(case["bias"])
        slots = torch.from_numpy(case["slots"])
        if spec["call"] == "decode":
            out = causal_conv1d_update(x, view, weight, bias, "silu", conv_state_indices=slots, validate_data=False)
        else:
            out = causal_conv1d_update(x, view, weight, bias, "silu", conv_state_indices=slots,
                                       num_accepted_tokens=torch.from_numpy(case["accepted"]),
                                       query_start_loc=torch.from_numpy(case["query_start_loc"]),
                                       max_query_len=spec["max_query_len"], validate_data=False)
        record = {"y": out.numpy(), "state": state.numpy()[np.unique(case["slots"])]}
        np.savez_compressed(HERE / f"{spec['name']}.npz", **record)
        print(spec["name"], {k: v.shape for k, v in record.items()})
    return 0


if __name__ == "__main__":
    sys.exit(main())
