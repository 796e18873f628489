/*
 * lightdelta_b200.h -- C ABI of the B200 (sm_100a) Gated DeltaNet decode hot path.
 *
 * Every entry point takes plain device pointers, element strides and sizes; no
 * framework types cross this boundary.  All entry points:
 *   - allocate nothing and never synchronise the host;
 *   - enqueue their kernels on `stream` (a cudaStream_t passed as void*; NULL is
 *     the legacy default stream), so a caller may capture them in a CUDA graph;
 *   - validate their arguments on the host first and return LD_ERR_INVALID with a
 *     message (ld_last_error) before touching the GPU when a precondition fails;
 *   - return LD_ERR_CUDA if the launch itself fails.
 * Data errors (a null or out-of-range slot, an accepted count outside the window)
 * never fault: the affected request is skipped as described per entry point, and
 * out-of-range slots additionally raise a bit in the device fault word
 * (ld_fault_flags).
 *
 * Geometry: key/value head dimension K = V = 128.  The state of one
 * (slot, value head) is a dense fp32 [V, K] matrix (row v, column k), 64 KiB.
 * A state slot is [HV, V, K]; slots sit `slot_stride` floats apart.
 */
#ifndef LIGHTDELTA_B200_H_
#define LIGHTDELTA_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. */
#define LD_OK 0
#define LD_ERR_INVALID 1 /* a host-checked precondition failed; nothing was launched */
#define LD_ERR_CUDA 2    /* the CUDA runtime reported an error */

/* Element types of the dtype-polymorphic parameters (dt_bias, norm weight). */
#define LD_DTYPE_F32 0
#define LD_DTYPE_BF16 1
#define LD_DTYPE_F16 2 /* ld_greedy_verify logits only */
#define LD_DTYPE_I32 3 /* token ids */
#define LD_DTYPE_I64 4 /* token ids */

/* Bits of the device fault word (ld_fault_flags). */
#define LD_FAULT_DECODE_SLOT_RANGE 0x1u   /* decode: a slot index >= n_slots */
#define LD_FAULT_DECODE_TOKENS 0x2u       /* decode: cu[r+1]-cu[r] > width, or cu outside [0, n_tokens] */
#define LD_FAULT_GATHER_SLOT_RANGE 0x4u   /* gather_state: a slot index >= n_pool_slots */
#define LD_FAULT_SCATTER_SLOT_RANGE 0x8u  /* scatter_state: a slot index >= n_pool_slots */
#define LD_FAULT_COPY_SLOT_RANGE 0x10u    /* copy_slots: a slot index >= n_pool_slots */
#define LD_FAULT_WAIT_TIMEOUT 0x20u       /* a bounded in-kernel wait expired: the CTA stored nothing more and returned */
#define LD_FAULT_VERIFY_DRAFTS 0x40u      /* greedy_verify: a request has more drafts than steps */
#define LD_FAULT_VERIFY_RANGE 0x80u       /* greedy_verify: metadata points outside the logits or token ids */
#define LD_FAULT_CONV_SLOT_RANGE 0x100u   /* conv update: a conv-state slot index >= n_conv_slots */

/* Head dimension handled by every kernel (K = V). */
#define LD_HEAD_DIM 128
/* Largest number of tokens per request (MTP verify window), csrc/register.cpp:5-7 schema
 * limit enforced at csrc/gdn_decode.cu:394-395. */
#define LD_MAX_WIDTH 4
/* Largest number of draft tokens per request in ld_greedy_verify (its sampled rows hold
 * num_speculative_steps + 1 tokens). */
#define LD_MAX_VERIFY_STEPS 7

/* Message of the last LD_ERR_* returned on the calling thread ("" if none). */
const char* ld_last_error(void);

/* Library version string. */
const char* ld_version(void);

/*
 * Fused GDN decode / MTP verify.
 * Replaces lightdelta::decode (csrc/gdn_decode.cu:360-420, declared at
 * include/lightdelta/ops.h:5-10, schema csrc/register.cpp:5-7).
 *
 * Requests r in [0, n_requests) own tokens cu[r] .. cu[r+1]-1 and a row of `width`
 * (1..4) int32 state slots indices[r*width + t].  For each (request, value head h):
 *   source slot  = indices[r*width + accepted[r]-1]   (accepted[r] in 1..width);
 *   S            = state[source, h]                    (fp32 [128,128]);
 *   for each token t:  S <- exp(g_t) S;  S <- S + beta_t (v_t - S k_t) k_t^T;
 *                      o_t = bf16(S q_t);  state[indices[r*width+t], h] <- S if that slot > 0;
 *   out[token, h, :] = bf16( o_t * rsqrt(mean(o_t^2)+eps) * weight * silu(gate[token,h,:]) ).
 * q and k are L2-normalised per head in fp32 (q additionally scaled by 128^-1/2);
 * g = -exp(a_log[h]) * softplus(a + dt_bias[h]); beta = sigmoid(b).
 * A request with no tokens writes nothing.  A request whose source slot is <= 0,
 * whose accepted count lies outside 1..width, whose token count exceeds width or whose
 * source slot is >= n_slots gets zero outputs and no state writes.
 * Destination slots <= 0 (and >= n_slots) are not written; slot 0 is therefore never
 * modified.
 *
 * qkv      bf16 rows [n_tokens, (2*H+HV)*128] = [q (H*128) | k (H*128) | v (HV*128)], row stride qkv_row_stride
 * a, b     bf16 [n_tokens, HV], row strides a_row_stride / b_row_stride, unit inner stride
 * a_log    fp32 [HV];  dt_bias [HV] of dt_bias_dtype;  weight [128] of weight_dtype
 * indices  int32 [n_requests, width] contiguous;  cu int32 [n_requests+1];  accepted int32 [n_requests]
 * state    fp32 [n_slots, HV, 128, 128], inner three dims dense, slot stride `slot_stride` floats
 * gate     bf16 [n_tokens, HV, 128], head stride 128, row stride gate_row_stride
 * out      bf16 [n_tokens, HV, 128] contiguous
 */
int ld_decode(const void* qkv, int64_t qkv_row_stride,
              const void* a, int64_t a_row_stride,
              const void* b, int64_t b_row_stride,
              const float* a_log,
              const void* dt_bias, int dt_bias_dtype,
              const int32_t* indices, int64_t n_requests, int64_t width,
              const int32_t* cu, const int32_t* accepted,
              float* state, int64_t n_slots, int64_t slot_stride,
              const void* gate, int64_t gate_row_stride,
              const void* weight, int weight_dtype,
              void* out, int64_t n_tokens,
              int64_t num_k_heads, int64_t num_v_heads,
              float eps, void* stream);

/*
 * Slot-indexed gather of whole state slots into a packed buffer.
 * Replaces lightdelta::gather_state (csrc/state_io.cu:44-58, include/lightdelta/ops.h:11-12,
 * schema csrc/register.cpp:8).
 *   out[i] = pool[slots[i*slots_stride]]   if that slot > 0 and valid[i] (and < n_pool_slots)
 *   out[i] = 0                             otherwise.
 * pool fp32, slot i at pool + slot*pool_slot_stride, `slot_elems` dense floats per slot;
 * out fp32 with row stride out_row_stride; valid: n bytes (C bool).
 */
int ld_gather_state(const float* pool, int64_t n_pool_slots, int64_t pool_slot_stride,
                    const int32_t* slots, int64_t slots_stride,
                    const uint8_t* valid, int64_t n,
                    float* out, int64_t out_row_stride,
                    int64_t slot_elems, void* stream);

/*
 * Slot-indexed scatter of a packed buffer into the pool.
 * Replaces lightdelta::scatter_state (csrc/state_io.cu:60-69, include/lightdelta/ops.h:13,
 * schema csrc/register.cpp:9).
 *   pool[slots[i*slots_stride]] = packed[i]   for every i whose slot is > 0 (and < n_pool_slots).
 * Rows whose slot is <= 0 are skipped, so slot 0 is never written.  Two rows naming the
 * same slot race (as in the reference).
 */
int ld_scatter_state(const float* packed, int64_t packed_row_stride,
                     const int32_t* slots, int64_t slots_stride, int64_t n,
                     float* pool, int64_t n_pool_slots, int64_t pool_slot_stride,
                     int64_t slot_elems, void* stream);

/*
 * Pool-to-pool slot copy: the explicit form of committing an accepted MTP step.
 * Extension with no single counterpart in the reference: it performs in one pass what
 * python/lightdelta/backend.py:87-91 (index_copy_ commit of live step states) does for a
 * state that already sits in the pool, i.e. gather_state followed by scatter_state.
 *   pool[dst[i]] = pool[src[i]]   for every i with src[i] > 0, dst[i] > 0 and src[i] != dst[i].
 * src/dst are int32 vectors with strides src_stride/dst_stride.  A slot named both as a
 * source and as a destination of different rows races.
 */
int ld_copy_slots(float* pool, int64_t n_pool_slots, int64_t pool_slot_stride,
                  const int32_t* src, int64_t src_stride,
                  const int32_t* dst, int64_t dst_stride, int64_t n,
                  int64_t slot_elems, void* stream);

/* Decode kernel variants (ld_decode_kernel_override). */
#define LD_DECODE_KERNEL_AUTO 0        /* library default: STREAM for width-1 launches of >= 9 items per SM (>= 7 with a bf16 pool), else ROWREG */
#define LD_DECODE_KERNEL_ROWREG 1      /* one CTA per (request, head), state loaded into registers */
#define LD_DECODE_KERNEL_STREAM 2      /* persistent kernel: TMA bulk loads into a 3-deep ring, 8 consumer warps */

/*
 * ld_decode on a bf16 state pool (state: bf16 [n_slots, HV, 128, 128], slot_stride elements, a
 * multiple of 8): each request's source state is widened to fp32, updated in fp32 across its
 * tokens exactly as ld_decode does, and every stored step is rounded to bf16 (nearest even).
 * Half the state bytes of an fp32 pool per token; results differ from the fp32 pool by that
 * rounding and, within fp32 rounding, by the order of the dot products' additions (each lane
 * owns eight consecutive bf16 columns).  One-token launches run a streaming kernel of their own
 * (two items in flight per CTA, state kept as packed bf16 words, q / k norms folded into the
 * reductions, so results also differ from the fp32 pool's in the last fp32 bits); multi-token
 * launches always run the one-CTA-per-item kernel (LD_DECODE_KERNEL_STREAM applies to one-token
 * launches only).  No counterpart in the reference, whose
 * launcher requires an fp32 pool (csrc/gdn_decode.cu:375-377).
 */
int ld_decode_bf16_state(const void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride,
                         const void* b, int64_t b_row_stride, const float* a_log, const void* dt_bias,
                         int dt_bias_dtype, const int32_t* indices, int64_t n_requests, int64_t width,
                         const int32_t* cu, const int32_t* accepted, void* state, int64_t n_slots,
                         int64_t slot_stride, const void* gate, int64_t gate_row_stride, const void* weight,
                         int weight_dtype, void* out, int64_t n_tokens, int64_t num_k_heads, int64_t num_v_heads,
                         float eps, void* stream);

/*
 * Causal depthwise conv1d state update of the q, k, v channels: vLLM's causal_conv1d_update as
 * python/lightdelta/integration/vllm_layer.py:161-172 (speculative decode: num_accepted_tokens,
 * query_start_loc, max_query_len) and :199-207 (one-token decode) call it.  No counterpart in
 * the reference, which calls vLLM's Triton kernel.
 *
 * x: [n_tokens, dim] bf16, rows x_row_stride elements apart; the post-conv activations replace
 *   the inputs in place (as vLLM does).
 * conv_state: bf16, element (slot, channel, position) at conv_state[slot * conv_slot_stride +
 *   channel * conv_dim_stride + position * conv_pos_stride] (vLLM's [slots, dim, L] storage and
 *   the transposed [slots, L, dim] one are both such views); conv_state_len = L >=
 *   conv_width - 2 + max_tokens.
 * conv_weight: [dim, conv_width] bf16 contiguous, 2 <= conv_width <= 4; conv_bias: [dim] bf16 or NULL.
 * Request r: conv slot slots[r * slots_stride] (0 = the null block: skipped), tokens
 *   [cu[r], cu[r+1]) (n <= max_tokens), window start accepted[r] - 1 (accepted NULL: 0).
 *   y_t = silu(bias + sum_j window_j * W[:, j] + x_t * W[:, w-1]) with the window shifting by
 *   one token per step (fp32 accumulator; bf16 x bf16 products rounded to bf16; y rounded to
 *   bf16); state positions [0, w - 2) take window positions [o + 1, o + w - 1), then
 *   [w - 2, w - 2 + n) take the inputs.
 * A conv slot >= n_conv_slots sets LD_FAULT_CONV_SLOT_RANGE; such requests, requests whose
 * tokens fall outside [0, n_tokens) (LD_FAULT_DECODE_TOKENS) and requests with accepted outside
 * [1, max_tokens] are left untouched.
 */
int ld_conv_update(void* x, int64_t x_row_stride, int64_t n_tokens, int64_t dim, void* conv_state,
                   int64_t n_conv_slots, int64_t conv_slot_stride, int64_t conv_dim_stride, int64_t conv_pos_stride,
                   int64_t conv_state_len, const void* conv_weight, const void* conv_bias, int64_t conv_width,
                   const int32_t* slots, int64_t slots_stride, const int32_t* accepted, const int32_t* cu,
                   int64_t n_requests, int64_t max_tokens, void* stream);

/*
 * The conv update followed by the GDN decode / MTP verify, as the vLLM layer runs them
 * (vllm_layer.py:161-174, :199-220), in one call: ld_conv_update on qkv with the conv slots
 * indices[r * width] (vLLM's conv_state_indices = slots[:, 0]), num_accepted_tokens = accepted
 * and max_tokens = width, then ld_decode on the post-conv qkv.  Arguments as the two; every one
 * is checked before anything is launched.  No counterpart in the reference.
 */
int ld_conv_decode(void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride, const void* b,
                   int64_t b_row_stride, const float* a_log, const void* dt_bias, int dt_bias_dtype,
                   const int32_t* indices, int64_t n_requests, int64_t width, const int32_t* cu,
                   const int32_t* accepted, float* state, int64_t n_slots, int64_t slot_stride, const void* gate,
                   int64_t gate_row_stride, const void* weight, int weight_dtype, void* out, int64_t n_tokens,
                   int64_t num_k_heads, int64_t num_v_heads, float eps, void* conv_state, int64_t n_conv_slots,
                   int64_t conv_slot_stride, int64_t conv_dim_stride, int64_t conv_pos_stride,
                   int64_t conv_state_len, const void* conv_weight, const void* conv_bias, int64_t conv_width,
                   void* stream);

/*
 * Process-wide choice of the kernel that ld_decode launches, for tuning and for testing every
 * variant against the oracle; all variants compute the same results.  The streaming kernel needs
 * 16-byte aligned qkv / gate rows and falls back to LD_DECODE_KERNEL_ROWREG otherwise.
 * Returns the previous setting, or -LD_ERR_INVALID for an unknown variant.
 * No counterpart in the reference, which has a single kernel (csrc/gdn_decode.cu:130).
 */
int ld_decode_kernel_override(int variant);

/*
 * Test hook of the persistent decode kernel's bounded waits, process-wide; no counterpart in the
 * reference.  Every mbarrier wait of that kernel gives up after limit_ns nanoseconds (0 restores
 * the default of one second), raises LD_FAULT_WAIT_TIMEOUT, and the CTA stops: it stores no state
 * or output of the item whose wait ran out or of any later item, waits (bounded) for the copies it
 * issued and returns.  extra_tx_bytes > 0 (at most 1024) makes every state load announce that many
 * bytes more than it copies, so the waits for it run out although every copy lands: a launch then
 * changes no pool slot and no output of a request it runs.  Settings apply to launches made after
 * the call.  Returns LD_OK, or LD_ERR_INVALID for arguments out of range.
 */
int ld_decode_wait_test(int64_t limit_ns, int32_t extra_tx_bytes);

/*
 * Programmatic dependent launch (PDL), process-wide: 1 (the default) launches every kernel
 * with programmatic stream serialisation, so its CTAs may be scheduled while the preceding
 * kernel on the stream finishes; each kernel waits (griddepcontrol.wait) for that kernel's
 * completion and memory before touching global memory, so results and ordering are unchanged.
 * 0 launches with plain stream order; -1 only queries.  Returns the previous setting.
 * No counterpart in the reference.
 */
int ld_programmatic_launch(int enable);

/*
 * Reads (and, if clear != 0, resets) the device fault word of the current device into *flags.
 * This call synchronises the device; it is a diagnostic, not part of the hot path.
 */
int ld_fault_flags(uint32_t* flags, int clear);

/*
 * Greedy MTP verification (the device form of the reference's rejection sampler,
 * python/lightdelta/runtime/speculation.py:274-326, LightDeltaRejectionSampler.__call__):
 *
 *   target = argmax over each logits row (first index of the maximum; NaN counts as the maximum)
 *   for each request r, with begin = cu_num_logits[r], end = cu_num_logits[r+1],
 *   d = num_draft_tokens[r] and drafts = input_ids[query_start_loc[r+1]-d, query_start_loc[r+1]):
 *     d == 0: sampled[r,0] = target[begin]; num_sampled[r] = 1 (0 for a prefill row)
 *     else:   accepted = length of the prefix with begin+i < end and target[begin+i] == drafts[i];
 *             sampled[r, 0..accepted) = drafts, sampled[r, accepted] = target[min(begin+accepted, end-1)];
 *             num_sampled[r] = accepted + 1 and num_rejected[r] = (end - begin) - (accepted + 1),
 *             both 0 for a prefill row (seq_lens[r] < prefill_len[r]).
 *   The remaining entries of sampled[r, 0..num_speculative_steps] are -1; num_rejected is 0
 *   where not set above.
 *
 * logits: [n_logits, vocab] of logits_dtype (F32, BF16 or F16), unit inner stride,
 *   logits_row_stride elements between rows.  Only the rows a request consults are read.
 * cu_num_logits, query_start_loc: int32 [n_requests + 1]; num_draft_tokens, seq_lens,
 *   prefill_len: int32 [n_requests].
 * input_ids: [n_input_ids] of token_dtype (I32 or I64); sampled: [n_requests,
 *   num_speculative_steps + 1] of token_dtype, row-major; num_sampled, num_rejected: int32
 *   [n_requests].  Every output entry is written.
 * Where the reference raises (d > num_speculative_steps) or indexes outside the logits or
 * input_ids, the request's row is -1 / 0 / 0 and LD_FAULT_VERIFY_DRAFTS or
 * LD_FAULT_VERIFY_RANGE is set in the fault word.
 * 0 <= num_speculative_steps <= LD_MAX_VERIFY_STEPS.
 */
int ld_greedy_verify(const void* logits, int logits_dtype, int64_t n_logits, int64_t vocab,
                     int64_t logits_row_stride, const int32_t* cu_num_logits, const int32_t* query_start_loc,
                     const void* input_ids, int token_dtype, int64_t n_input_ids, const int32_t* num_draft_tokens,
                     const int32_t* seq_lens, const int32_t* prefill_len, int64_t n_requests,
                     int64_t num_speculative_steps, void* sampled, int32_t* num_sampled, int32_t* num_rejected,
                     void* stream);

/*
 * Process-wide thread-block cluster size of ld_greedy_verify (0 = automatic, or 1, 2, 4, 8, 16
 * CTAs per request), for tuning and tests; results do not depend on it.  Returns the previous
 * setting, or -LD_ERR_INVALID for another value.  No counterpart in the reference.
 */
int ld_greedy_verify_cluster_override(int cluster);

/* Size of the static device scratch of ld_decode_packed_noalloc (64 MiB on every GPU that loads
 * the library, held until the process exits): 32 KiB of per-call request plan, then the fp32
 * scratch state slots. */
#define LD_NOALLOC_SCRATCH_BYTES (64LL * 1024 * 1024)

/*
 * Packed-mode decode / MTP verify that allocates nothing.  It has no counterpart in the
 * reference; it exists for callers that cannot allocate device memory while they decode: a host
 * that binds this C ABI from a runtime with no device allocator of its own, an engine that hands
 * the whole GPU to its state pools at start-up and forbids later allocations, or a latency-bound
 * loop that cannot afford cudaMalloc's implicit device-wide synchronisation.
 *
 * Arguments, results and errors are those of ld_decode (state = the fp32 pool).  It computes what
 * the packed state path computes (python/lightdelta/backend.py:30-91): each request's source state
 * is gathered into a scratch slot, decoded there, and every live step state is committed to its
 * pool slot (null destinations skipped).  Outputs and pool contents equal ld_decode's.
 * The scratch is one static device array of LD_NOALLOC_SCRATCH_BYTES:
 *   - it must hold (1 + n_requests * width) slots of num_v_heads * 64 KiB after its 32 KiB plan
 *     region (at num_v_heads = 32: n_requests * width <= 30), and n_requests * width <= 1024;
 *     larger calls return LD_ERR_INVALID with a message, before any launch;
 *   - the first call on each device looks up the array's device address (cudaGetSymbolAddress
 *     with that device current) and keeps it; make that first call before any stream capture;
 *   - every call overwrites the parts it reads, so nothing needs clearing between calls, but all
 *     calls on a device share the array: calls whose work overlaps on the GPU (other streams,
 *     other host threads) race and corrupt each other's results.
 * No cudaMalloc, cudaFree or other allocating routine is called.
 */
int ld_decode_packed_noalloc(const void* qkv, int64_t qkv_row_stride, const void* a, int64_t a_row_stride,
                             const void* b, int64_t b_row_stride, const float* a_log, const void* dt_bias,
                             int dt_bias_dtype, const int32_t* indices, int64_t n_requests, int64_t width,
                             const int32_t* cu, const int32_t* accepted, float* state, int64_t n_slots,
                             int64_t slot_stride, const void* gate, int64_t gate_row_stride, const void* weight,
                             int weight_dtype, void* out, int64_t n_tokens, int64_t num_k_heads,
                             int64_t num_v_heads, float eps, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* LIGHTDELTA_B200_H_ */
