"""GPU parity of torch.ops.lightdelta.greedy_verify / ld_greedy_verify (the device form of
python/lightdelta/runtime/speculation.py:274-326) against the reference's golden outputs and
the CPU oracle: bit-exact token ids and counts for every logits dtype, token dtype, cluster size
and layout, plus the fault paths and CUDA-graph replay."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from golden import cases

pytestmark = pytest.mark.gpu

GOLDEN = cases.__file__.rsplit("/", 1)[0]
TORCH_DTYPES = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def device_logits(spec_dtype, values: np.ndarray, device) -> torch.Tensor:
    return torch.from_numpy(values).to(device).to(TORCH_DTYPES[spec_dtype])


def oracle_logits(spec_dtype, logits: torch.Tensor) -> np.ndarray:
    if spec_dtype == "bf16":
        return logits.cpu().view(torch.int16).numpy().view(np.uint16)
    return logits.cpu().numpy()


def run_device(logits, case, steps, token_dtype, device, via="op"):
    meta = {k: torch.from_numpy(np.asarray(case[k], np.int32)).to(device)
            for k in ("cu_num_logits", "query_start_loc", "num_draft_tokens", "seq_lens", "prefill_len")}
    input_ids = torch.from_numpy(np.asarray(case["input_ids"], np.int64)).to(device).to(token_dtype)
    n = meta["num_draft_tokens"].numel()
    sampled = torch.full((n, steps + 1), 12345, dtype=token_dtype, device=device)
    num_sampled = torch.full((n,), 777, dtype=torch.int32, device=device)
    num_rejected = torch.full((n,), 777, dtype=torch.int32, device=device)
    args = (logits, meta["cu_num_logits"], meta["query_start_loc"], input_ids, meta["num_draft_tokens"],
            meta["seq_lens"], meta["prefill_len"], sampled, num_sampled, num_rejected)
    if via == "op":
        torch.ops.lightdelta.greedy_verify(*args)
    else:
        from lightdelta_b200 import capi

        capi.greedy_verify(*args)
    torch.cuda.synchronize()
    return sampled.cpu().to(torch.int64).numpy(), num_sampled.cpu().numpy(), num_rejected.cpu().numpy()


def expect_oracle(logits, case, steps, spec_dtype):
    return oracle.greedy_verify(oracle_logits(spec_dtype, logits), case["cu_num_logits"], case["query_start_loc"],
                                case["input_ids"], case["num_draft_tokens"], case["seq_lens"], case["prefill_len"],
                                steps)


def assert_same(got, want):
    np.testing.assert_array_equal(got[0], want[0])
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[2], want[2])


@pytest.fixture
def cluster(native):
    def force(q):
        native.set_verify_cluster(q)

    yield force
    native.set_verify_cluster(0)


@pytest.mark.parametrize("via", ["op", "capi"])
def test_known_answer_of_the_reference_test(device, via):
    """tests/test_runtime.py:7-23 on the device."""
    logits = torch.full((6, 40), -100.0, device=device)
    for row, token in enumerate([10, 11, 12, 20, 31, 32]):
        logits[row, token] = 1
    case = dict(cu_num_logits=[0, 3, 6], query_start_loc=[0, 2, 4], input_ids=[10, 11, 20, 21],
                num_draft_tokens=[2, 2], seq_lens=[4, 4], prefill_len=[0, 0])
    sampled, num_sampled, num_rejected = run_device(logits, case, 2, torch.int64, device, via)
    assert sampled.tolist() == [[10, 11, 12], [20, 31, -1]]
    assert num_sampled.tolist() == [3, 2]
    assert num_rejected.tolist() == [0, 1]


@pytest.mark.parametrize("q", [0, 1, 2, 4, 8])
@pytest.mark.parametrize("spec", cases.SAMPLER_CASES, ids=lambda s: s["name"])
def test_matches_reference_golden(device, cluster, spec, q):
    cluster(q)
    case = cases.sampler_case(spec)
    golden = np.load(f"{GOLDEN}/{spec['name']}.npz")
    logits = device_logits(spec["dtype"], case["logits"], device)
    token_dtype = torch.int64 if spec["tokens"] == "i64" else torch.int32
    got = run_device(logits, case, spec["steps"], token_dtype, device)
    assert_same(got, (golden["sampled"], golden["num_sampled"], golden["num_rejected"]))


@pytest.mark.parametrize("dtype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("layout", ["padded_rows", "odd_offset"])
def test_strided_and_unaligned_logits(device, cluster, dtype, layout):
    """Rows inside a wider buffer (16-byte aligned rows, vector path) and rows starting one
    element into it (scalar path)."""
    cluster(4)
    spec = dict(cases.SAMPLER_CASES[0])
    case = cases.sampler_case(spec)
    values = torch.from_numpy(case["logits"]).to(device)
    n, vocab = values.shape
    pad = 3 if layout == "padded_rows" else 4  # 2053 + 3: rows 16-byte aligned for every dtype
    wide = torch.full((n, vocab + pad), float("inf"), device=device).to(TORCH_DTYPES[dtype])
    start = 0 if layout == "padded_rows" else 1
    logits = wide[:, start:start + vocab]
    logits.copy_(values.to(TORCH_DTYPES[dtype]))
    got = run_device(logits, case, spec["steps"], torch.int32, device)
    want = expect_oracle(logits, case, spec["steps"], dtype)
    assert want[3] == 0
    assert_same(got, want)


def full_size_case(requests=64, steps=3, vocab=151936, seed=21):
    """BASELINE config-3-shaped verification: 64 requests x 3 drafts x 4 logits rows."""
    rng = np.random.default_rng(seed)
    drafts = np.full(requests, steps, np.int32)
    rows = drafts + 1
    cu = np.concatenate([[0], np.cumsum(rows)]).astype(np.int32)
    qsl = np.concatenate([[0], np.cumsum(drafts + 1)]).astype(np.int32)
    input_ids = rng.integers(0, vocab, int(qsl[-1]))
    logits = rng.standard_normal((int(cu[-1]), vocab), dtype=np.float32)
    accepted = rng.integers(0, steps + 1, requests)
    for r in range(requests):
        draft = input_ids[qsl[r + 1] - steps: qsl[r + 1]]
        for i in range(rows[r]):
            token = draft[i] if i < accepted[r] else rng.integers(0, vocab)
            logits[cu[r] + i, token] = 8.0
    return logits, dict(cu_num_logits=cu, query_start_loc=qsl, input_ids=input_ids, num_draft_tokens=drafts,
                        seq_lens=np.full(requests, 100, np.int32), prefill_len=np.zeros(requests, np.int32))


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_full_size_matches_oracle(device, dtype):
    values, case = full_size_case()
    logits = device_logits(dtype, values, device)
    got = run_device(logits, case, 3, torch.int32, device)
    want = expect_oracle(logits, case, 3, dtype)
    assert want[3] == 0
    assert_same(got, want)
    assert got[1].sum() > len(got[1])  # some drafts were accepted


def test_fault_paths(device, native):
    native.fault_flags(clear=True)
    logits = torch.zeros(4, 64, device=device)
    logits[:, 7] = 1.0
    case = dict(cu_num_logits=[0, 1, 2, 9, 10], query_start_loc=[0, 2, 4, 6, 99], input_ids=[7, 7, 7, 7, 7, 7],
                num_draft_tokens=[3, 1, 1, 2], seq_lens=[9, 9, 9, 9], prefill_len=[0, 0, 0, 0])
    got = run_device(logits, case, 2, torch.int32, device)
    want = expect_oracle(logits, case, 2, "f32")
    assert_same(got, want)
    flags = native.fault_flags(clear=True)
    assert flags == want[3] == native.LD_FAULT_VERIFY_DRAFTS | native.LD_FAULT_VERIFY_RANGE
    assert got[0][0].tolist() == [-1, -1, -1] and got[0][3].tolist() == [-1, -1, -1]
    assert native.fault_flags(clear=True) == 0


def test_sampler_class_on_a_reference_style_batch(device):
    from lightdelta_b200.sampler import LightDeltaRejectionSampler

    spec = cases.SAMPLER_CASES[1]
    case = cases.sampler_case(spec)
    golden = np.load(f"{GOLDEN}/{spec['name']}.npz")
    batch = SimpleNamespace(
        num_reqs=spec["requests"],
        num_draft_tokens_per_req=case["num_draft_tokens"],  # host numpy, as vLLM passes it
        input_ids=torch.from_numpy(case["input_ids"]).to(device).to(torch.int32),
        query_start_loc=torch.from_numpy(case["query_start_loc"]).to(device),
        cu_num_logits=torch.from_numpy(case["cu_num_logits"]).to(device),
        seq_lens=torch.from_numpy(case["seq_lens"]).to(device),
        prefill_len_np=case["prefill_len"],
    )
    output = LightDeltaRejectionSampler(spec["steps"])(device_logits(spec["dtype"], case["logits"], device), batch)
    assert output.sampled_token_ids.dtype == torch.int32
    np.testing.assert_array_equal(output.sampled_token_ids.cpu().numpy(), golden["sampled"])
    np.testing.assert_array_equal(output.num_sampled.cpu().numpy(), golden["num_sampled"])
    np.testing.assert_array_equal(output.num_rejected.cpu().numpy(), golden["num_rejected"])


def test_graph_replay_with_new_logits(device):
    values, case = full_size_case(requests=16, vocab=32000, seed=3)
    logits = torch.from_numpy(values).to(device)
    meta = {k: torch.from_numpy(np.asarray(case[k], np.int32)).to(device)
            for k in ("cu_num_logits", "query_start_loc", "num_draft_tokens", "seq_lens", "prefill_len")}
    input_ids = torch.from_numpy(np.asarray(case["input_ids"], np.int32)).to(device)
    sampled = torch.empty(16, 4, dtype=torch.int32, device=device)
    num_sampled = torch.empty(16, dtype=torch.int32, device=device)
    num_rejected = torch.empty_like(num_sampled)

    def step():
        torch.ops.lightdelta.greedy_verify(logits, meta["cu_num_logits"], meta["query_start_loc"], input_ids,
                                           meta["num_draft_tokens"], meta["seq_lens"], meta["prefill_len"],
                                           sampled, num_sampled, num_rejected)

    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        step()
    torch.cuda.current_stream().wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        step()
    for seed in (5, 6):
        new_values, _ = full_size_case(requests=16, vocab=32000, seed=seed)
        logits.copy_(torch.from_numpy(new_values))
        graph.replay()
        torch.cuda.synchronize()
        want = expect_oracle(logits, case, 3, "f32")
        assert_same((sampled.cpu().to(torch.int64).numpy(), num_sampled.cpu().numpy(), num_rejected.cpu().numpy()),
                    want)


def test_no_requests_is_a_no_op(device):
    logits = torch.zeros(0, 16, device=device)
    empty = torch.zeros(0, dtype=torch.int32, device=device)
    one = torch.zeros(1, dtype=torch.int32, device=device)
    sampled = torch.zeros(0, 4, dtype=torch.int32, device=device)
    torch.ops.lightdelta.greedy_verify(logits, one, one, empty, empty, empty, empty, sampled, empty, empty)
    torch.cuda.synchronize()
