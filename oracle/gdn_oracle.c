/*
 * gdn_oracle.c -- CPU restatement of LightDelta's GDN decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the lightdelta_b200
 * CUDA kernels and the timed CPU baseline of bench.py.  It is never linked into, loaded
 * by or called from the product path (lightdelta_b200/).
 *
 * It restates, in plain C with fp32 arithmetic:
 *   oracle_post_conv_gdn  python/lightdelta/reference/gdn.py:70-128 (post_conv_gdn), for any
 *                         head counts and head dimensions, with optional per-step checkpoints;
 *   oracle_decode         the pool-indexed decode / MTP-verify contract of lightdelta::decode
 *                         (csrc/gdn_decode.cu:130-354 semantics, driven as in
 *                         python/lightdelta/backend.py:24-28), whose packed form is
 *                         python/lightdelta/backend.py:30-91;
 *   oracle_gather_state / oracle_scatter_state
 *                         csrc/state_io.cu:11-27 (+ launchers :44-69);
 *   oracle_copy_slots     the one-pass pool-to-pool commit (backend.py:87-91 applied to states
 *                         already in the pool).
 * Element-wise operations follow the reference order (e.g. decayed = S*decay, then
 * decayed + delta*k with two roundings; build with -ffp-contract=off); reductions use eight
 * partial sums, which differs from torch's reduction order only by fp32 rounding.
 * bf16 values are passed as their raw uint16 bit patterns and rounded to nearest-even.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define ORACLE_DIM 128

static inline float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof(f));
  return f;
}

static inline uint16_t f32_to_bf16(float f) {
  uint32_t u;
  memcpy(&u, &f, sizeof(u));
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u); /* quiet NaN */
  u += 0x7fffu + ((u >> 16) & 1u);                                            /* nearest-even */
  return (uint16_t)(u >> 16);
}

static inline float round_bf16(float f) { return bf16_to_f32(f32_to_bf16(f)); }

/* Sum of x[i]*y[i] over n elements with eight partial sums (vectorisable without reassociation). */
static float dot(const float* x, const float* y, int64_t n) {
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  int64_t i = 0;
  for (; i + 8 <= n; i += 8) {
    for (int l = 0; l < 8; ++l) acc[l] += x[i + l] * y[i + l];
  }
  for (int l = 0; i < n; ++i, ++l) acc[l] += x[i] * y[i];
  return ((acc[0] + acc[1]) + (acc[2] + acc[3])) + ((acc[4] + acc[5]) + (acc[6] + acc[7]));
}

/* torch.nn.functional.softplus, beta 1, threshold 20. */
static inline float softplus(float x) { return x > 20.0f ? x : log1pf(expf(x)); }
static inline float sigmoid(float x) { return 1.0f / (1.0f + expf(-x)); }
static inline float silu(float x) { return x / (1.0f + expf(-x)); }

/* q <- q * rsqrt(sum(q^2) + 1e-6) [* scale]: gdn.py:98-101. */
static void l2_normalise(float* x, int64_t n, int apply_scale, float scale) {
  const float inv = 1.0f / sqrtf(dot(x, x, n) + 1e-6f);
  for (int64_t i = 0; i < n; ++i) {
    x[i] = x[i] * inv;
    if (apply_scale) x[i] = x[i] * scale;
  }
}

/* One delta-rule step on a [V,K] state (gdn.py:111-114); updates S only if live. */
static void delta_step(float* S, int64_t V, int64_t K, const float* kn, const float* v, float decay, float beta,
                       int live, float* scratch) {
  if (!live) return;
  for (int64_t row = 0; row < V; ++row) {
    float* s = S + row * K;
    for (int64_t i = 0; i < K; ++i) scratch[i] = s[i] * decay;
    const float prediction = dot(scratch, kn, K);
    const float delta = (v[row] - prediction) * beta;
    for (int64_t i = 0; i < K; ++i) s[i] = scratch[i] + delta * kn[i];
  }
}

/* Output of one step: raw = S q (rounded to bf16 if io_bf16), gated RMSNorm (gdn.py:115-119). */
static void step_output(const float* S, int64_t V, int64_t K, const float* qn, const float* gate,
                        const float* norm_weight, float eps, int io_bf16, int live, float* raw, float* out) {
  float square = 0.0f;
  for (int64_t row = 0; row < V; ++row) {
    float r = dot(S + row * K, qn, K);
    if (io_bf16) r = round_bf16(r);
    raw[row] = r;
  }
  square = dot(raw, raw, V);
  const float rstd = 1.0f / sqrtf(square / (float)V + eps);
  for (int64_t row = 0; row < V; ++row) {
    float y = live ? raw[row] * rstd * norm_weight[row] * silu(gate[row]) : 0.0f;
    if (io_bf16) y = round_bf16(y);
    out[row] = y;
  }
}

static void set_threads(int threads) {
#ifdef _OPENMP
  if (threads > 0) omp_set_num_threads(threads);
#else
  (void)threads;
#endif
}

/*
 * post_conv_gdn (gdn.py:70-128).  All tensors are dense row-major fp32 values:
 *   q, k [B,T,Hk,K]; v, gate [B,T,Hv,V]; a, b [B,T,Hv]; a_log, dt_bias [Hv]; norm_weight [V];
 *   initial_state [B,Hv,V,K]; lengths [B].
 * Outputs: output [B,T,Hv,V]; final_state [B,Hv,V,K]; checkpoints [B,T+1,Hv,V,K] or NULL.
 * io_bf16 != 0 reproduces bf16 activations: the recurrence output and the final output are
 * rounded to bf16 (gdn.py:116, :120).  Returns 0, or -1 on invalid geometry.
 */
int oracle_post_conv_gdn(int64_t B, int64_t T, int64_t Hk, int64_t Hv, int64_t K, int64_t V, const float* q,
                         const float* k, const float* v, const float* a, const float* b, const float* a_log,
                         const float* dt_bias, const float* gate, const float* norm_weight,
                         const float* initial_state, const int64_t* lengths, int io_bf16, float norm_eps,
                         float* output, float* final_state, float* checkpoints, int threads) {
  if (B <= 0 || T <= 0 || Hk <= 0 || Hv <= 0 || K <= 0 || V <= 0 || Hv % Hk != 0 || !(norm_eps > 0.0f)) return -1;
  const int64_t ratio = Hv / Hk;
  const float scale = (float)pow((double)K, -0.5);
  const int64_t state_elems = V * K;
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t pair = 0; pair < B * Hv; ++pair) {
    const int64_t bi = pair / Hv, h = pair % Hv, kh = h / ratio;
    float* S = (float*)malloc(sizeof(float) * (size_t)(state_elems + 2 * K + 2 * V + K));
    float* qn = S + state_elems;
    float* kn = qn + K;
    float* raw = kn + K;
    float* out_row = raw + V;
    float* scratch = out_row + V;
    memcpy(S, initial_state + (bi * Hv + h) * state_elems, sizeof(float) * (size_t)state_elems);
    if (checkpoints) memcpy(checkpoints + ((bi * (T + 1)) * Hv + h) * state_elems, S, sizeof(float) * (size_t)state_elems);
    const float g_scale = -expf(a_log[h]);
    for (int64_t t = 0; t < T; ++t) {
      const int live = lengths[bi] > t;
      const int64_t bt = bi * T + t;
      memcpy(qn, q + (bt * Hk + kh) * K, sizeof(float) * (size_t)K);
      memcpy(kn, k + (bt * Hk + kh) * K, sizeof(float) * (size_t)K);
      l2_normalise(qn, K, 1, scale);
      l2_normalise(kn, K, 0, 1.0f);
      const float decay = expf(g_scale * softplus(a[bt * Hv + h] + dt_bias[h]));
      const float beta = sigmoid(b[bt * Hv + h]);
      delta_step(S, V, K, kn, v + (bt * Hv + h) * V, decay, beta, live, scratch);
      step_output(S, V, K, qn, gate + (bt * Hv + h) * V, norm_weight, norm_eps, io_bf16, live, raw, out_row);
      memcpy(output + (bt * Hv + h) * V, out_row, sizeof(float) * (size_t)V);
      if (checkpoints) {
        memcpy(checkpoints + ((bi * (T + 1) + t + 1) * Hv + h) * state_elems, S, sizeof(float) * (size_t)state_elems);
      }
    }
    memcpy(final_state + (bi * Hv + h) * state_elems, S, sizeof(float) * (size_t)state_elems);
    free(S);
  }
  return 0;
}

/*
 * Pool-indexed decode / MTP verify: the contract of lightdelta::decode
 * (csrc/gdn_decode.cu:130-354), with the same argument meaning as ld_decode.
 *   request r: tokens cu[r]..cu[r+1]-1, slots indices[r*W .. r*W+W-1];
 *   source = indices[r*W + accepted[r]-1]; step t's state -> indices[r*W+t] if > 0.
 * Invalid requests (no valid source, n > W, source >= n_slots) get zero outputs and no
 * writes; a request with no tokens is skipped (gdn_decode.cu:150-168).
 * state_bf16 selects a bf16 pool (no counterpart in the reference, whose pool is fp32): the
 * source head is widened to fp32, the recurrence runs in fp32 across the request's tokens, and
 * each stored step is rounded to bf16 (nearest even).
 * Returns 0, or -1 on invalid arguments.
 */
static void load_head(const void* state, int state_bf16, int64_t at, float* S, int64_t n) {
  if (!state_bf16) {
    memcpy(S, (const float*)state + at, sizeof(float) * (size_t)n);
    return;
  }
  const uint16_t* src = (const uint16_t*)state + at;
  for (int64_t i = 0; i < n; ++i) S[i] = bf16_to_f32(src[i]);
}

static void store_head(void* state, int state_bf16, int64_t at, const float* S, int64_t n) {
  if (!state_bf16) {
    memcpy((float*)state + at, S, sizeof(float) * (size_t)n);
    return;
  }
  uint16_t* dst = (uint16_t*)state + at;
  for (int64_t i = 0; i < n; ++i) dst[i] = f32_to_bf16(S[i]);
}

int oracle_decode_state(const uint16_t* qkv, int64_t qkv_row, const uint16_t* a, int64_t a_row, const uint16_t* b,
                        int64_t b_row, const float* a_log, const void* dt_bias, int dt_bias_bf16,
                        const int32_t* indices, int64_t R, int64_t W, const int32_t* cu, const int32_t* accepted,
                        void* state, int state_bf16, int64_t n_slots, int64_t slot_stride, const uint16_t* gate,
                        int64_t gate_row, const void* weight, int weight_bf16, uint16_t* out, int64_t n_tokens,
                        int64_t H, int64_t HV, float eps, int threads) {
  const int64_t D = ORACLE_DIM;
  if (W < 1 || W > 4 || H <= 0 || HV <= 0 || HV % H != 0 || !(eps > 0.0f)) return -1;
  const int64_t ratio = HV / H;
  const int64_t head_elems = D * D;
  const float scale = (float)pow((double)D, -0.5);
  float weight_f[ORACLE_DIM];
  for (int64_t i = 0; i < D; ++i) {
    weight_f[i] = weight_bf16 ? bf16_to_f32(((const uint16_t*)weight)[i]) : ((const float*)weight)[i];
  }
  set_threads(threads);
#pragma omp parallel for schedule(dynamic, 1)
  for (int64_t pair = 0; pair < R * HV; ++pair) {
    const int64_t r = pair / HV, h = pair % HV, kh = h / ratio;
    const int64_t bos = cu[r], eos = cu[r + 1], n = eos - bos;
    if (n <= 0) continue;
    if (bos < 0 || eos > n_tokens) continue;
    const int64_t acc = accepted[r];
    const int64_t src = (acc >= 1 && acc <= W) ? indices[r * W + acc - 1] : 0;
    if (src <= 0 || n > W || src >= n_slots) {
      for (int64_t t = 0; t < n; ++t) memset(out + ((bos + t) * HV + h) * D, 0, sizeof(uint16_t) * (size_t)D);
      continue;
    }
    float* S = (float*)malloc(sizeof(float) * (size_t)(head_elems + 6 * D));
    float *qn = S + head_elems, *kn = qn + D, *vv = kn + D, *z = vv + D, *raw = z + D, *out_row = raw + D;
    float scratch[ORACLE_DIM];
    load_head(state, state_bf16, src * slot_stride + h * head_elems, S, head_elems);
    const float g_scale = -expf(a_log[h]);
    const float dt = dt_bias_bf16 ? bf16_to_f32(((const uint16_t*)dt_bias)[h]) : ((const float*)dt_bias)[h];
    for (int64_t t = 0; t < n; ++t) {
      const int64_t token = bos + t;
      const uint16_t* row = qkv + token * qkv_row;
      for (int64_t i = 0; i < D; ++i) {
        qn[i] = bf16_to_f32(row[kh * D + i]);
        kn[i] = bf16_to_f32(row[(H + kh) * D + i]);
        vv[i] = bf16_to_f32(row[(2 * H + h) * D + i]);
        z[i] = bf16_to_f32(gate[token * gate_row + h * D + i]);
      }
      l2_normalise(qn, D, 1, scale);
      l2_normalise(kn, D, 0, 1.0f);
      const float decay = expf(g_scale * softplus(bf16_to_f32(a[token * a_row + h]) + dt));
      const float beta = sigmoid(bf16_to_f32(b[token * b_row + h]));
      delta_step(S, D, D, kn, vv, decay, beta, 1, scratch);
      step_output(S, D, D, qn, z, weight_f, eps, 1, 1, raw, out_row);
      for (int64_t i = 0; i < D; ++i) out[(token * HV + h) * D + i] = f32_to_bf16(out_row[i]);
      const int64_t dst = indices[r * W + t];
      if (dst > 0 && dst < n_slots) {
        store_head(state, state_bf16, dst * slot_stride + h * head_elems, S, head_elems);
      }
    }
    free(S);
  }
  return 0;
}

int oracle_decode(const uint16_t* qkv, int64_t qkv_row, const uint16_t* a, int64_t a_row, const uint16_t* b,
                  int64_t b_row, const float* a_log, const void* dt_bias, int dt_bias_bf16, const int32_t* indices,
                  int64_t R, int64_t W, const int32_t* cu, const int32_t* accepted, float* state, int64_t n_slots,
                  int64_t slot_stride, const uint16_t* gate, int64_t gate_row, const void* weight, int weight_bf16,
                  uint16_t* out, int64_t n_tokens, int64_t H, int64_t HV, float eps, int threads) {
  return oracle_decode_state(qkv, qkv_row, a, a_row, b, b_row, a_log, dt_bias, dt_bias_bf16, indices, R, W, cu,
                             accepted, state, 0, n_slots, slot_stride, gate, gate_row, weight, weight_bf16, out,
                             n_tokens, H, HV, eps, threads);
}

/* gather_state (csrc/state_io.cu:11-27, :44-58): out[i] = live ? pool[slot] : 0. */
void oracle_gather_state(const float* pool, int64_t n_pool_slots, int64_t pool_stride, const int32_t* slots,
                         int64_t slots_stride, const uint8_t* valid, int64_t n, float* out, int64_t out_stride,
                         int64_t slot_elems, int threads) {
  set_threads(threads);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) {
    const int64_t slot = slots[i * slots_stride];
    float* dst = out + i * out_stride;
    if (slot > 0 && slot < n_pool_slots && valid[i]) {
      memcpy(dst, pool + slot * pool_stride, sizeof(float) * (size_t)slot_elems);
    } else {
      memset(dst, 0, sizeof(float) * (size_t)slot_elems);
    }
  }
}

/* scatter_state (csrc/state_io.cu:11-27, :60-69): pool[slot] = packed[i] for slot > 0, in row order. */
void oracle_scatter_state(const float* packed, int64_t packed_stride, const int32_t* slots, int64_t slots_stride,
                          int64_t n, float* pool, int64_t n_pool_slots, int64_t pool_stride, int64_t slot_elems) {
  for (int64_t i = 0; i < n; ++i) {
    const int64_t slot = slots[i * slots_stride];
    if (slot <= 0 || slot >= n_pool_slots) continue;
    memcpy(pool + slot * pool_stride, packed + i * packed_stride, sizeof(float) * (size_t)slot_elems);
  }
}

/* One-pass commit: pool[dst[i]] = pool[src[i]] for src, dst > 0 and src != dst, in row order. */
void oracle_copy_slots(float* pool, int64_t n_pool_slots, int64_t pool_stride, const int32_t* src,
                       int64_t src_stride, const int32_t* dst, int64_t dst_stride, int64_t n, int64_t slot_elems) {
  for (int64_t i = 0; i < n; ++i) {
    const int64_t from = src[i * src_stride], to = dst[i * dst_stride];
    if (from <= 0 || to <= 0 || from == to || from >= n_pool_slots || to >= n_pool_slots) continue;
    memcpy(pool + to * pool_stride, pool + from * pool_stride, sizeof(float) * (size_t)slot_elems);
  }
}
