/*
 * conv_oracle.c -- CPU restatement of the causal depthwise conv1d state update that feeds the
 * GDN decode (vLLM's causal_conv1d_update, as LightDelta's vLLM layer calls it).
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for lightdelta_b200's fused
 * conv + decode operator.  It is never linked into, loaded by or called from the product path.
 *
 * The algorithm lives in a third-party dependency: vLLM, pinned at 0.29.0 by the reference
 * (requirements/lock-cu129.txt:202), called at python/lightdelta/integration/vllm_layer.py:161-172
 * (speculative decode: num_accepted_tokens, query_start_loc, max_query_len = indices width) and
 * :199-207 (one-token decode).  vLLM 0.29.0 is not in this image; the restatement follows the
 * published causal_conv1d_update of the vLLM release that is (0.22), whose speculative-decode
 * path takes the same arguments.  Per request r with conv slot c = slots[r] (skipped when c is
 * the null block 0), tokens [qsl[r], qsl[r+1]) (n of them, none: skipped), offset
 * o = accepted[r] - 1 and kernel width w:
 *   window  col_j = state[c, :, o + j], j < w - 1
 *   output  y_t = silu(bias + sum_j col_j * W[:, j] + x_t * W[:, w-1]), then the window shifts
 *           left by one and takes x_t
 *   state   new[:, t] = state[c, :, o + 1 + t] for t < w - 2, then x_0 .. x_{n-1}
 *           (w - 2 + n positions written, the rest of the slot untouched)
 * Arithmetic follows the Triton kernel: the accumulator is fp32 and starts at the bias; each
 * product of two bf16 operands is rounded to bf16 before it is added (Triton's bf16 x bf16
 * product is bf16); silu is acc / (1 + exp(-acc)) in fp32; y is rounded to the state dtype.
 * With an fp32 state the products are plain fp32.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

static float bf16_bits_to_f32(uint16_t h) {
  const uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof(f));
  return f;
}

static uint16_t f32_to_bf16_bits(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof(u));
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

static float round_bf16(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }

/* Element access for the two state dtypes: 0 = f32, 1 = bf16 bits. */
static float get(const void* base, int dtype, int64_t at) {
  return dtype == 0 ? ((const float*)base)[at] : bf16_bits_to_f32(((const uint16_t*)base)[at]);
}

static void put(void* base, int dtype, int64_t at, float v) {
  if (dtype == 0) {
    ((float*)base)[at] = v;
  } else {
    ((uint16_t*)base)[at] = f32_to_bf16_bits(v);
  }
}

/*
 * x:        [n_tokens, dim] of state_dtype, row stride x_row (elements); read only
 * y:        [n_tokens, dim] of state_dtype, row stride y_row; post-conv values (rows of skipped
 *           requests receive x unchanged)
 * state:    conv state of state_dtype, element (slot, channel, position) at
 *           slot * s_slot + channel * s_dim + position * s_pos; updated in place
 * weight:   [dim, width] of weight_dtype (0 = f32, 1 = bf16), contiguous; bias [dim] or NULL
 * slots:    conv slot per request (stride slots_stride); accepted, qsl as described above
 * Returns 0, or -1 for invalid arguments.
 */
int oracle_conv_update(const void* x, int64_t x_row, void* y, int64_t y_row, void* state, int state_dtype,
                       int64_t n_state_slots, int64_t s_slot, int64_t s_dim, int64_t s_pos, int64_t state_len,
                       const void* weight, int weight_dtype, const void* bias, int64_t dim, int64_t width,
                       const int32_t* slots, int64_t slots_stride, const int32_t* accepted, const int32_t* qsl,
                       int64_t n_requests, int64_t n_tokens) {
  if (width < 2 || width > 6 || dim <= 0) return -1;
  for (int64_t t = 0; t < n_tokens; ++t) {
    for (int64_t c = 0; c < dim; ++c) put(y, state_dtype, t * y_row + c, get(x, state_dtype, t * x_row + c));
  }
  float window[8];
  for (int64_t r = 0; r < n_requests; ++r) {
    const int64_t slot = slots[r * slots_stride];
    if (slot == 0) continue; /* null block */
    if (slot < 0 || slot >= n_state_slots) return -1;
    const int64_t begin = qsl[r], end = qsl[r + 1];
    const int64_t n = end - begin;
    if (n <= 0) continue;
    if (begin < 0 || end > n_tokens) return -1;
    const int64_t offset = (int64_t)accepted[r] - 1;
    const int64_t written = width - 2 + n;
    if (offset < 0 || offset + width - 1 > state_len || written > state_len) return -1;
    for (int64_t c = 0; c < dim; ++c) {
      const int64_t base = slot * s_slot + c * s_dim;
      for (int64_t j = 0; j < width - 1; ++j) window[j] = get(state, state_dtype, base + (offset + j) * s_pos);
      float shifted[8];
      for (int64_t t = 0; t < width - 2; ++t) shifted[t] = get(state, state_dtype, base + (offset + 1 + t) * s_pos);
      const float b = bias == NULL ? 0.0f : get(bias, weight_dtype, c);
      float wts[8];
      for (int64_t j = 0; j < width; ++j) wts[j] = get(weight, weight_dtype, c * width + j);
      for (int64_t t = 0; t < n; ++t) {
        const float xt = get(x, state_dtype, (begin + t) * x_row + c);
        float acc = b;
        for (int64_t j = 0; j < width; ++j) {
          const float v = j < width - 1 ? window[j] : xt;
          float prod = v * wts[j];
          if (state_dtype == 1 && weight_dtype == 1) prod = round_bf16(prod);
          acc = acc + prod;
        }
        for (int64_t j = 0; j + 1 < width - 1; ++j) window[j] = window[j + 1];
        window[width - 2] = xt;
        const float out = acc / (1.0f + expf(-acc));
        put(y, state_dtype, (begin + t) * y_row + c, out);
      }
      for (int64_t t = 0; t < width - 2; ++t) put(state, state_dtype, base + t * s_pos, shifted[t]);
      for (int64_t t = 0; t < n; ++t) {
        put(state, state_dtype, base + (width - 2 + t) * s_pos, get(x, state_dtype, (begin + t) * x_row + c));
      }
    }
  }
  return 0;
}
