"""CPU tests of greedy MTP verification (python/lightdelta/runtime/speculation.py:274-326):
the oracle against the reference's known-answer test and golden fixtures made by the reference
itself, the C ABI's host-side checks, and the host-side rules of the drop-in sampler class.
Nothing here launches a kernel."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

import oracle
from golden import cases, detrand

GOLDEN = cases.__file__.rsplit("/", 1)[0]


def oracle_logits(spec, logits):
    if spec["dtype"] == "bf16":
        return detrand.bf16_bits(logits)
    if spec["dtype"] == "f16":
        return logits.astype(np.float16)
    return logits


def test_known_answer_of_the_reference_test():
    """tests/test_runtime.py:7-23 restated on the oracle."""
    logits = np.full((6, 40), -100.0, np.float32)
    for row, token in enumerate([10, 11, 12, 20, 31, 32]):
        logits[row, token] = 1
    sampled, num_sampled, num_rejected, faults = oracle.greedy_verify(
        logits, [0, 3, 6], [0, 2, 4], [10, 11, 20, 21], [2, 2], [4, 4], [0, 0], 2)
    assert sampled.tolist() == [[10, 11, 12], [20, 31, -1]]
    assert num_sampled.tolist() == [3, 2]
    assert num_rejected.tolist() == [0, 1]
    assert faults == 0


@pytest.mark.parametrize("spec", cases.SAMPLER_CASES, ids=lambda s: s["name"])
def test_oracle_matches_reference_golden(spec):
    case = cases.sampler_case(spec)
    golden = np.load(f"{GOLDEN}/{spec['name']}.npz")
    logits = oracle_logits(spec, case["logits"])
    np.testing.assert_array_equal(oracle.argmax_rows(logits), golden["target"])
    sampled, num_sampled, num_rejected, faults = oracle.greedy_verify(
        logits, case["cu_num_logits"], case["query_start_loc"], case["input_ids"], case["num_draft_tokens"],
        case["seq_lens"], case["prefill_len"], spec["steps"])
    assert faults == 0
    np.testing.assert_array_equal(sampled, golden["sampled"])
    np.testing.assert_array_equal(num_sampled, golden["num_sampled"])
    np.testing.assert_array_equal(num_rejected, golden["num_rejected"])


@pytest.mark.parametrize("dtype", [np.float32, np.float16, "bf16"])
def test_oracle_argmax_follows_torch(dtype):
    rng = np.random.default_rng(5)
    values = np.round(rng.standard_normal((64, 257)) * 2) / 2  # many exact ties
    values[3, 17] = np.nan
    values[3, 9] = np.nan
    values[4, :] = -np.inf
    values[5, 100] = np.inf
    values[6, :] = np.nan
    values = values.astype(np.float32)
    if dtype == "bf16":
        bits = detrand.bf16_bits(values)
        expected = torch.from_numpy(bits.view(np.int16)).view(torch.bfloat16).argmax(-1).numpy()
        got = oracle.argmax_rows(bits)
    else:
        array = values.astype(dtype)
        expected = torch.from_numpy(array).argmax(-1).numpy()
        got = oracle.argmax_rows(array)
    np.testing.assert_array_equal(got, expected)


def test_oracle_flags_too_many_drafts_and_out_of_range_rows():
    logits = np.zeros((4, 8), np.float32)
    sampled, num_sampled, num_rejected, faults = oracle.greedy_verify(
        logits, [0, 2, 9], [0, 4, 6], [1, 2, 3, 4, 5, 6], [3, 2], [5, 5], [0, 0], 2)
    assert faults == oracle.VERIFY_FAULT_DRAFTS | oracle.VERIFY_FAULT_RANGE
    assert sampled.tolist() == [[-1, -1, -1], [-1, -1, -1]]
    assert num_sampled.tolist() == [0, 0] and num_rejected.tolist() == [0, 0]


def test_capi_rejects_bad_arguments_before_touching_the_gpu(native):
    lib = native.lib()
    args = [None, native.LD_DTYPE_F32, 4, 8, 8, None, None, None, native.LD_DTYPE_I32, 4, None, None, None, 2, 3,
            None, None, None, None]
    bad_steps = list(args)
    bad_steps[14] = native.MAX_VERIFY_STEPS + 1
    assert lib.ld_greedy_verify(*bad_steps) == native.LD_ERR_INVALID
    assert "num_speculative_steps" in native.last_error()
    bad_stride = list(args)
    bad_stride[4] = 7
    assert lib.ld_greedy_verify(*bad_stride) == native.LD_ERR_INVALID
    bad_dtype = list(args)
    bad_dtype[1] = 9
    assert lib.ld_greedy_verify(*bad_dtype) == native.LD_ERR_INVALID
    assert lib.ld_greedy_verify(*args) == native.LD_ERR_INVALID  # NULL pointers
    empty = list(args)
    empty[13] = 0
    assert lib.ld_greedy_verify(*empty) == native.LD_OK  # no requests: nothing to do
    assert lib.ld_greedy_verify_cluster_override(3) == -native.LD_ERR_INVALID
    assert lib.ld_greedy_verify_cluster_override(0) == 0


def test_sampler_class_keeps_the_reference_host_errors(native):
    from lightdelta_b200.sampler import LightDeltaRejectionSampler

    batch = SimpleNamespace(num_reqs=1, num_draft_tokens_per_req=np.array([3]), input_ids=torch.zeros(4),
                            query_start_loc=torch.tensor([0, 4]), cu_num_logits=torch.tensor([0, 4]),
                            seq_lens=torch.tensor([4]), prefill_len_np=np.array([0]))
    with pytest.raises(ValueError, match="draft logits"):
        LightDeltaRejectionSampler(2)(torch.zeros(4, 8), batch, draft_logits=torch.zeros(1))
    with pytest.raises(ValueError, match="invalid MTP draft-token metadata"):
        LightDeltaRejectionSampler(2)(torch.zeros(4, 8), batch)
