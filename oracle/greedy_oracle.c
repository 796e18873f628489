/*
 * greedy_oracle.c -- CPU restatement of LightDelta's greedy MTP verification.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for lightdelta_b200's
 * greedy_verify kernel and the timed CPU baseline of bench.py's sampling workload.  It is
 * never linked into, loaded by or called from the product path (lightdelta_b200/).
 *
 * It restates python/lightdelta/runtime/speculation.py:274-326
 * (LightDeltaRejectionSampler.__call__):
 *   oracle_argmax_rows    target = logits.argmax(dim=-1) (speculation.py:279) with torch's
 *                         order: the first index of the maximum, NaN counted as the maximum;
 *   oracle_greedy_verify  the per-request prefix check of speculation.py:292-325.
 * Where the reference raises (more drafts than steps, speculation.py:305-306) or would index
 * outside the logits or the token ids, the request's outputs are -1 / 0 / 0 and a fault bit
 * is returned instead (0x40 drafts, 0x80 range), which is what the device kernel does.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define VERIFY_FAULT_DRAFTS 0x40u
#define VERIFY_FAULT_RANGE 0x80u

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h >> 15) << 31;
  const uint32_t exponent = (h >> 10) & 0x1fu;
  uint32_t mantissa = h & 0x3ffu;
  uint32_t bits;
  if (exponent == 0x1fu) {
    bits = sign | 0x7f800000u | (mantissa << 13);
  } else if (exponent != 0) {
    bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
  } else if (mantissa == 0) {
    bits = sign;
  } else { /* subnormal: normalise */
    uint32_t e = 113;
    while ((mantissa & 0x400u) == 0) {
      mantissa <<= 1;
      --e;
    }
    bits = sign | (e << 23) | ((mantissa & 0x3ffu) << 13);
  }
  float f;
  memcpy(&f, &bits, sizeof(f));
  return f;
}

static float logit_at(const void* logits, int dtype, int64_t at) {
  if (dtype == 0) return ((const float*)logits)[at];
  const uint16_t raw = ((const uint16_t*)logits)[at];
  if (dtype == 1) {
    const uint32_t bits = (uint32_t)raw << 16;
    float f;
    memcpy(&f, &bits, sizeof(f));
    return f;
  }
  return half_to_float(raw);
}

/* target[i] = argmax of row i; dtype 0 = f32, 1 = bf16 bits, 2 = f16 bits. */
void oracle_argmax_rows(const void* logits, int dtype, int64_t n_rows, int64_t vocab, int64_t row_stride,
                        int64_t* target, int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#pragma omp parallel for schedule(static)
#endif
  for (int64_t i = 0; i < n_rows; ++i) {
    const int64_t base = i * row_stride;
    float best = logit_at(logits, dtype, base);
    int64_t index = 0;
    if (!isnan(best)) {
      for (int64_t j = 1; j < vocab; ++j) {
        const float v = logit_at(logits, dtype, base + j);
        if (isnan(v)) {
          index = j;
          break;
        }
        if (v > best) {
          best = v;
          index = j;
        }
      }
    }
    target[i] = index;
  }
}

/* Returns the fault bits; outputs as ld_greedy_verify. */
uint32_t oracle_greedy_verify(const void* logits, int dtype, int64_t n_logits, int64_t vocab, int64_t row_stride,
                              const int32_t* cu_num_logits, const int32_t* query_start_loc, const int64_t* input_ids,
                              int64_t n_input_ids, const int32_t* num_draft_tokens, const int32_t* seq_lens,
                              const int32_t* prefill_len, int64_t n_requests, int64_t steps, int64_t* sampled,
                              int32_t* num_sampled, int32_t* num_rejected, int64_t* target, int threads) {
  oracle_argmax_rows(logits, dtype, n_logits, vocab, row_stride, target, threads);
  uint32_t faults = 0;
  for (int64_t r = 0; r < n_requests; ++r) {
    int64_t* row = sampled + r * (steps + 1);
    for (int64_t c = 0; c <= steps; ++c) row[c] = -1;
    num_sampled[r] = 0;
    num_rejected[r] = 0;
    const int64_t begin = cu_num_logits[r], end = cu_num_logits[r + 1];
    const int64_t drafts = num_draft_tokens[r];
    const int prefill = seq_lens[r] < prefill_len[r];
    if (drafts > steps) {
      faults |= VERIFY_FAULT_DRAFTS;
      continue;
    }
    /* Rows the request may consult: [begin, min(begin + drafts, end - 1)], or end - 1 alone
     * when it has no logits, or begin alone without drafts. */
    int64_t lo, hi;
    if (drafts == 0) {
      lo = hi = begin;
    } else if (end > begin) {
      lo = begin;
      hi = begin + (drafts > 0 ? drafts : 0);
      if (hi > end - 1) hi = end - 1;
    } else {
      lo = hi = end - 1;
    }
    if (lo < 0 || hi >= n_logits) {
      faults |= VERIFY_FAULT_RANGE;
      continue;
    }
    if (drafts == 0) { /* speculation.py:295-302 */
      row[0] = target[begin];
      num_sampled[r] = prefill ? 0 : 1;
      continue;
    }
    const int64_t input_end = query_start_loc[r + 1];
    int64_t accepted = 0;
    int bad = 0;
    while (accepted < drafts) { /* speculation.py:307-312 */
      if (begin + accepted >= end) break;
      const int64_t at = input_end - drafts + accepted;
      if (at < 0 || at >= n_input_ids) {
        bad = 1;
        break;
      }
      if (target[begin + accepted] != input_ids[at]) break;
      row[accepted] = input_ids[at];
      ++accepted;
    }
    if (bad) {
      for (int64_t c = 0; c <= steps; ++c) row[c] = -1;
      faults |= VERIFY_FAULT_RANGE;
      continue;
    }
    int64_t bonus = begin + accepted; /* speculation.py:313-314 */
    if (bonus > end - 1) bonus = end - 1;
    row[accepted] = target[bonus];
    if (!prefill) { /* speculation.py:315-325 */
      num_sampled[r] = (int32_t)(accepted + 1);
      num_rejected[r] = (int32_t)((end - begin) - (accepted + 1));
    }
  }
  return faults;
}
