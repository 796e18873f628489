"""Case definitions shared by tests/golden/make_golden.py and the tests that read the fixtures.

Every input is regenerated from its seed with tests/golden/detrand.py, so the fixtures hold
only results.  Distributions follow the reference's test fixture (tests/conftest.py:5-33:
qkvz*0.2, ba ~ N(0,1), pool*0.1, bf16 dt_bias and norm weight) and, for the HV=32 cases, the
BASELINE configs (q, k, v ~ N(0,1); a_log = dt_bias = 0 so g = -softplus(a); state ~ N(0, 0.02^2);
gate 0.2*N(0,1)).
"""

from __future__ import annotations

import numpy as np

from . import detrand

D = 128

POST_CONV_CASES = [
    # The reference's own odd-shape case (tests/test_gdn.py:7-44): fp32 io, lengths [4,2,0].
    dict(name="post_conv_small", seed=7, B=3, T=4, Hk=2, Hv=6, K=5, V=7, io_bf16=False, checkpoints=True,
         lengths=[4, 2, 0], eps=1e-6, samples=None, baseline=False),
    # B=1, T=1, H=16, HV=32, K=V=128, bf16 activations.
    dict(name="post_conv_hv32_t1", seed=11, B=1, T=1, Hk=16, Hv=32, K=D, V=D, io_bf16=True, checkpoints=False,
         lengths=[1], eps=1e-6, samples=32768, baseline=True),
    # MTP-shaped multi-step run with per-step checkpoints and one short request.
    dict(name="post_conv_hv32_t4", seed=13, B=2, T=4, Hk=16, Hv=32, K=D, V=D, io_bf16=True, checkpoints=True,
         lengths=[4, 2], eps=1e-6, samples=65536, baseline=True),
    # HV=48 geometry with non-zero a_log / dt_bias and a masked (length 0) request.
    dict(name="post_conv_hv48_t3", seed=17, B=2, T=3, Hk=16, Hv=48, K=D, V=D, io_bf16=True, checkpoints=False,
         lengths=[3, 0], eps=1e-5, samples=32768, baseline=False),
]

BACKEND_CASES = [
    # tests/test_gdn.py:58-75: mixed accepted counts, one padding request (slots[-1] = 0).
    *[dict(name=f"backend_hv48_w{w}", seed=42, batch=4, width=w, mutation="mixed", samples_per_slot=256)
      for w in (1, 2, 3, 4)],
    # tests/test_gdn.py:105-122: ragged tokens, invalid request, discarded candidate slot.
    dict(name="backend_hv48_ragged", seed=42, batch=4, width=4, mutation="ragged", samples_per_slot=256),
    # tests/test_gdn.py:78-102: flipped slot rows and accepted = 2.
    dict(name="backend_hv48_flipped", seed=42, batch=2, width=3, mutation="flipped", samples_per_slot=256),
]


SAMPLER_CASES = [
    # Greedy MTP verification (speculation.py:274-326): mixed draft counts, short logits spans,
    # a request without logits, prefill rows, ties, NaN / +-inf rows; int64 tokens as in the
    # reference's own test (tests/test_runtime.py:7-23).
    dict(name="sampler_f32_mixed", seed=101, requests=48, steps=3, vocab=2053, dtype="f32", tokens="i64",
         ties_per_row=1),
    # bf16 logits with several equal maxima per row and int32 tokens (vLLM's input_ids dtype).
    dict(name="sampler_bf16_ties", seed=103, requests=32, steps=3, vocab=4096, dtype="bf16", tokens="i32",
         ties_per_row=3),
    # fp16 logits, seven draft tokens (LD_MAX_VERIFY_STEPS), odd vocabulary.
    dict(name="sampler_f16_steps7", seed=107, requests=20, steps=7, vocab=1537, dtype="f16", tokens="i32",
         ties_per_row=1),
    # Qwen3 vocabulary size: the argmax spans several CTAs of a cluster.
    dict(name="sampler_f32_vocab151936", seed=109, requests=12, steps=3, vocab=151936, dtype="f32", tokens="i32",
         ties_per_row=1),
]


CONV_CASES = [
    # Speculative decode as vllm_layer.py:161-172 calls it: ragged tokens per request (0..4), a
    # null conv slot, accepted counts 1..4, bias; state [slots, dim, L] with L = 3 + 3.
    dict(name="conv_spec_dimfirst", seed=201, requests=10, width=4, max_query_len=4, dim=640, slots=24,
         layout="dim_first", bias=True, call="spec"),
    # The same on a token-first state (the transposed view vllm_layer.py:146-147 makes).
    dict(name="conv_spec_tokenfirst", seed=203, requests=10, width=4, max_query_len=4, dim=640, slots=24,
         layout="token_first", bias=False, call="spec"),
    # One-token decode as vllm_layer.py:199-207 calls it (no accepted counts, 2-D x) on a state
    # sized for speculative decode.
    dict(name="conv_decode_tokens1", seed=207, requests=12, width=4, max_query_len=1, dim=512, slots=20,
         layout="dim_first", bias=False, call="decode", state_len=6),
    # Kernel width 3.
    dict(name="conv_spec_width3", seed=209, requests=8, width=3, max_query_len=3, dim=384, slots=16,
         layout="dim_first", bias=True, call="spec"),
]


def spec_by_name(name: str) -> dict:
    for spec in POST_CONV_CASES + BACKEND_CASES + SAMPLER_CASES + CONV_CASES:
        if spec["name"] == name:
            return spec
    raise KeyError(name)


def sample_positions(seed: int, size: int, samples: int | None) -> np.ndarray:
    if samples is None or samples >= size:
        return np.arange(size, dtype=np.int64)
    return np.unique(detrand.integers(seed, samples, size))


def per_slot_positions(seed: int, shape, per_slot: int) -> np.ndarray:
    slots = shape[0]
    elems = int(np.prod(shape[1:]))
    rows = [s * elems + np.unique(detrand.integers(seed + s, per_slot, elems)) for s in range(slots)]
    return np.concatenate(rows).astype(np.int64)


def post_conv_inputs(spec: dict) -> dict:
    """fp32 arrays (already rounded to bf16 where the case uses bf16 activations)."""
    B, T, Hk, Hv, K, V = (spec[k] for k in ("B", "T", "Hk", "Hv", "K", "V"))
    s = spec["seed"] * 16

    def act(seed, shape, scale=1.0):
        values = detrand.normal(seed, shape, scale)
        return detrand.bf16_values(detrand.bf16_bits(values)) if spec["io_bf16"] else values

    arrays = dict(
        q=act(s + 1, (B, T, Hk, K)),
        k=act(s + 2, (B, T, Hk, K)),
        v=act(s + 3, (B, T, Hv, V)),
        a=act(s + 4, (B, T, Hv)),
        b=act(s + 5, (B, T, Hv)),
        gate=act(s + 8, (B, T, Hv, V), 0.2 if spec["baseline"] else 1.0),
    )
    if spec["baseline"]:
        arrays["a_log"] = np.zeros(Hv, np.float32)
        arrays["dt_bias"] = np.zeros(Hv, np.float32)
        arrays["initial_state"] = detrand.normal(s + 9, (B, Hv, V, K), 0.02)
    else:
        arrays["a_log"] = detrand.normal(s + 6, (Hv,))
        arrays["dt_bias"] = detrand.normal(s + 7, (Hv,))
        arrays["initial_state"] = detrand.normal(s + 9, (B, Hv, V, K))
    arrays["norm_weight"] = detrand.normal(s + 10, (V,))
    arrays["lengths"] = np.asarray(spec["lengths"], np.int64)
    return arrays


def backend_case(spec: dict) -> dict:
    """Inputs of a GDNBackend call at the reference geometry (H=16, HV=48), as numpy arrays.

    bf16 tensors are uint16 bit arrays: qkvz [n,16384] (qkv = [:, :10240], gate = [:, 10240:]),
    ba [n,96] (b = [:, :48], a = [:, 48:]) exactly as the reference fixture slices them.
    """
    batch, width = spec["batch"], spec["width"]
    n = batch * width
    hv, h = 48, 16
    qkv_width = (2 * h + hv) * D
    s = spec["seed"] * 10
    arrays = dict(
        qkvz_bits=detrand.bf16_bits(detrand.normal(s + 1, (n, qkv_width + hv * D), 0.2)),
        ba_bits=detrand.bf16_bits(detrand.normal(s + 2, (n, 2 * hv))),
        a_log=detrand.normal(s + 3, (hv,)),
        dt_bias_bits=detrand.bf16_bits(detrand.normal(s + 4, (hv,))),
        pool=detrand.normal(s + 5, (n + 2, hv, D, D), 0.1),
        weight_bits=detrand.bf16_bits(detrand.normal(s + 6, (D,))),
        slots=np.arange(1, n + 1, dtype=np.int32).reshape(batch, width),
        cu=np.arange(0, n + 1, width, dtype=np.int32),
        accepted=np.ones(batch, np.int32),
    )
    rows = n
    if spec["mutation"] == "mixed":
        arrays["accepted"][:] = np.arange(batch) % width + 1
        arrays["slots"][-1] = 0
    elif spec["mutation"] == "ragged":
        arrays["cu"] = np.array([0, 4, 7, 8, 8], np.int32)
        arrays["accepted"][0] = 0
        arrays["slots"][1, 2] = 0
        rows = 8
    elif spec["mutation"] == "flipped":
        arrays["slots"] = np.ascontiguousarray(arrays["slots"][::-1])
        arrays["accepted"][:] = 2
    else:
        raise ValueError(spec["mutation"])
    return dict(arrays=arrays, rows=rows, hv=hv, h=h, qkv_width=qkv_width)


def sampler_case(spec: dict) -> dict:
    """Inputs of a LightDeltaRejectionSampler call (speculation.py:274-326) as numpy arrays.

    logits are float32 values already rounded to the case's dtype ("f32", "bf16", "f16");
    cu_num_logits / query_start_loc / num_draft_tokens / seq_lens / prefill_len are int32,
    input_ids int64 (cast to the case's token dtype by the caller).  Each request's logits
    rows plant the draft tokens as the row maximum for a seeded accepted prefix, then a
    mismatch; some rows add equal maxima (ties), NaN or +-inf.
    """
    R, steps, vocab = spec["requests"], spec["steps"], spec["vocab"]
    s = spec["seed"] * 100
    u = lambda k, n: detrand.uniform(s + k, n)  # noqa: E731
    drafts = detrand.integers(s + 1, R, steps + 1)
    short = u(2, R) < 0.15
    rows = np.where(short & (drafts > 0), drafts, drafts + 1)
    if R > 5:  # a request with drafts but no logits rows: the bonus comes from target[end - 1]
        drafts[5], rows[5] = 2, 0
    accepted = (u(3, R) * (drafts + 1)).astype(np.int64)
    extra_inputs = np.where(u(4, R) < 0.25, 2, 0)
    inputs = drafts + 1 + extra_inputs
    seq_lens = 1 + detrand.integers(s + 5, R, 1000)
    prefill = u(6, R) < 0.2
    prefill_len = np.where(prefill, seq_lens + 1, 0)

    query_start_loc = np.concatenate([[0], np.cumsum(inputs)]).astype(np.int32)
    input_ids = detrand.integers(s + 7, int(inputs.sum()), vocab)
    cu = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    n_logits = int(cu[-1]) + 3  # three trailing rows that no request consults
    logits = detrand.normal(s + 8, (n_logits, vocab))

    total_rows = n_logits
    planted_random = detrand.integers(s + 9, total_rows, vocab)
    shift = 1 + detrand.integers(s + 10, total_rows, vocab - 1)
    tie_pos = detrand.integers(s + 11, total_rows * max(1, spec["ties_per_row"]), vocab).reshape(total_rows, -1)
    row_kind = u(12, total_rows)
    special_pos = detrand.integers(s + 13, total_rows, vocab)
    for r in range(R):
        draft = input_ids[query_start_loc[r + 1] - drafts[r]: query_start_loc[r + 1]]
        for i in range(rows[r]):
            row = cu[r] + i
            if i < accepted[r] and i < drafts[r]:
                token = draft[i]
            elif i < drafts[r]:
                token = (draft[i] + shift[row]) % vocab
            else:
                token = planted_random[row]
            logits[row, token] = 6.0
    for row in range(total_rows):
        kind = row_kind[row]
        if kind < 0.25:  # equal maxima: the first index wins
            logits[row, tie_pos[row]] = logits[row].max()
        elif kind < 0.31:
            logits[row, special_pos[row]] = np.nan
        elif kind < 0.34:
            logits[row, :] = -np.inf
        elif kind < 0.37:
            logits[row, special_pos[row]] = np.inf
    if spec["dtype"] == "bf16":
        logits = detrand.bf16_values(detrand.bf16_bits(logits))
    elif spec["dtype"] == "f16":
        logits = logits.astype(np.float16).astype(np.float32)
    return dict(
        logits=logits.astype(np.float32),
        cu_num_logits=cu,
        query_start_loc=query_start_loc,
        input_ids=input_ids.astype(np.int64),
        num_draft_tokens=drafts.astype(np.int32),
        seq_lens=seq_lens.astype(np.int32),
        prefill_len=prefill_len.astype(np.int32),
    )


def conv_case(spec: dict) -> dict:
    """Inputs of one causal_conv1d_update call (fp32 numpy arrays and int32 metadata).

    state is returned in its storage layout: [slots, dim, L] for "dim_first", [slots, L, dim]
    for "token_first" (the caller passes the [slots, dim, L] transposed view).
    """
    R, W, width, dim, S = (spec[k] for k in ("requests", "max_query_len", "width", "dim", "slots"))
    L = spec.get("state_len", width - 1 + W - 1)
    s = spec["seed"] * 100
    if spec["call"] == "decode":
        lengths = np.ones(R, np.int64)
        accepted = np.ones(R, np.int64)
    else:
        lengths = detrand.integers(s + 1, R, W + 1)  # 0..W tokens
        lengths[0] = W
        accepted = 1 + detrand.integers(s + 2, R, W)
    qsl = np.concatenate([[0], np.cumsum(lengths)]).astype(np.int32)
    slots = (1 + np.argsort(detrand.uniform(s + 3, S - 1), kind="stable")[:R]).astype(np.int32)  # distinct
    if R > 3:
        slots[3] = 0  # null block: the request is skipped
    shape = (S, dim, L) if spec["layout"] == "dim_first" else (S, L, dim)
    return dict(
        x=detrand.normal(s + 4, (int(qsl[-1]), dim)),
        state=detrand.normal(s + 5, shape),
        weight=detrand.normal(s + 6, (dim, width), 0.5),
        bias=detrand.normal(s + 7, (dim,), 0.1) if spec["bias"] else None,
        slots=slots,
        accepted=accepted.astype(np.int32),
        query_start_loc=qsl,
    )


def conv_state_view(spec: dict, state: np.ndarray) -> np.ndarray:
    """[slots, dim, L] view of a conv_case state array."""
    return state if spec["layout"] == "dim_first" else state.transpose(0, 2, 1)
