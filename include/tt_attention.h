/*
 * tt_attention.h - C ABI of the sm_100a (B200) BF16 causal attention forward.
 *
 * Plain C: raw device pointers, element strides and sizes, a CUDA stream passed as
 * `void*` (a cudaStream_t / CUstream), and an integer status. No allocation happens
 * behind these entry points: the caller owns O, LSE and the workspace.
 *
 * Each entry point names the reference interface it replaces (Tiny-transformer,
 * paths relative to that project).
 *
 * Device selection: call with the device that owns the pointers current on the
 * calling thread (cudaSetDevice, or a torch CUDAGuard), as for any CUDA library.
 */
#ifndef TT_ATTENTION_H_
#define TT_ATTENTION_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TT_ATTN_API __attribute__((visibility("default")))
#else
#define TT_ATTN_API
#endif

#define TT_ATTN_ABI_VERSION 1
#define TT_ATTN_HEAD_DIM 64

typedef enum tt_attn_status {
  TT_ATTN_OK = 0,
  TT_ATTN_BAD_ARG = 1,     /* invalid sizes, pointers or strides; nothing was launched */
  TT_ATTN_UNSUPPORTED = 2, /* valid request this path cannot take (layout, device);
                              nothing was launched: copy to an aligned contiguous layout */
  TT_ATTN_LAUNCH_FAIL = 3, /* a CUDA call failed; tt_attn_last_error() has the CUDA message */
  TT_ATTN_TIMEOUT = 4      /* a kernel wait ran out (see tt_attn_device_status) */
} tt_attn_status;

/*
 * Causal attention forward, BF16 in / BF16 O / FP32 LSE, head_dim 64.
 *
 * Replaces the BF16 branch of `attention_forward(q, k, v, past_len, segment_ids)`
 * (csrc/attention/attention.cu:32-159, declared in csrc/attention/attention.h:7-9,
 * bound in csrc/attention/bindings.cpp:4-8), i.e. the kernels
 * attention_bf16::forward<EVEN_TILES> (attention_forward_BF16_kernel.cuh:232-389) and
 * decode_partial / decode_merge (attention_decode_BF16_kernel.cuh:45-128).
 *
 *   q        [batch, heads, q_len, 64]  bf16, element strides q_strides[4]
 *   k, v     [batch, heads, kv_len, 64] bf16, element strides k_strides / v_strides
 *            (prefix views of a larger KV cache are read in place)
 *   past_len must equal kv_len - q_len; key j is visible to query row i iff j <= i + past_len.
 *   kv_lens  optional device int32[batch] (q_len must be 1): key j is visible iff
 *            j < kv_lens[b]; values are clamped to [0, kv_len]; 0 gives O = 0, LSE = -inf.
 *   out      contiguous [batch, heads, q_len, 64] bf16
 *   lse      contiguous [batch, heads, q_len] fp32, natural log
 *   workspace / workspace_bytes: device scratch of at least
 *            tt_attn_forward_workspace_size(...) bytes (may be NULL when that is 0). Decode
 *            (q_len == 1) of more than 2^20 (batch * heads * kv_len) K/V rows (2^21 when
 *            batch * heads <= 640) keeps a work
 *            counter and per-sequence arrival counters there, which the call zeroes on
 *            `stream` before its kernel runs, and its split-KV partials; prefill with fewer
 *            256-row query blocks than SMs keeps the partial records of its split blocks.
 *   stream   cudaStream_t the kernels are launched on; no host synchronisation.
 *
 * Layout requirements (else TT_ATTN_UNSUPPORTED): last stride 1, other strides positive
 * multiples of 8 elements, base pointers 16-byte aligned.
 */
TT_ATTN_API tt_attn_status tt_attn_forward_bf16(
    const void* q, const int64_t* q_strides,
    const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides,
    int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int64_t head_dim,
    int64_t past_len, const int32_t* kv_lens,
    void* out, float* lse,
    void* workspace, size_t workspace_bytes,
    void* stream);

/* Scratch bytes tt_attn_forward_bf16 needs for this shape: for decode of a cache longer than
 * 1024 keys, a 256-byte work counter, plus (when sequences are split into more than one chunk)
 * one 4-byte arrival counter per (batch, head) rounded up to 256 bytes and 272 bytes of FP32
 * partial per (batch, head, chunk). Replaces the partials tensor the reference allocates
 * (attention.cu:128-129). Returns 0 for decode of caches of up to 1024 keys (one CTA per
 * sequence, no scratch), for prefill shapes and for invalid shapes. */
TT_ATTN_API size_t tt_attn_forward_workspace_size(int64_t batch, int64_t heads, int64_t q_len,
                                                  int64_t kv_len);

/* 1 when a [.., .., .., 64] bf16 operand at `ptr` with these element strides can be read
 * in place; 0 when it must first be copied to aligned contiguous storage.
 * Replaces the alignment decision of aligned_contiguous (attention.cu:20-29). */
TT_ATTN_API int tt_attn_layout_supported(const void* ptr, const int64_t* strides);

/* 1 when the current device can run the kernels (compute capability 10.x), else 0.
 * Replaces the SM80 capability check (attention.cu:72-73). */
TT_ATTN_API int tt_attn_device_supported(void);

/* Reads (and, when clear != 0, resets) the current device's kernel status bits:
 * bit 0 = a bounded wait inside a kernel ran out (returns TT_ATTN_TIMEOUT);
 * bit 1 = tt_rope_append_bf16 met a device-held position outside the cache or the table and
 * skipped those rows (returns TT_ATTN_BAD_ARG). Synchronises the device. */
TT_ATTN_API tt_attn_status tt_attn_device_status(unsigned* flags, int clear);

/*
 * BF16 causal attention backward: dQ, dK, dV from the forward's inputs, output O and LSE.
 *
 * Replaces `attention_backward(q, k, v, dO, O, lse, past_len, segment_ids)`
 * (csrc/attention/attention.cu:161-234, declared in csrc/attention/attention.h, bound in
 * csrc/attention/bindings.cpp), i.e. the preprocess, dKdV and dQ kernels
 * (attention_backward_preprocess_kernel.cuh, attention_backward_dKdV_kernel.cu,
 * attention_backward_dQ_kernel.cu). Same arithmetic: D = rowsum(dO * O), P = exp(S / 8 - LSE),
 * dS = P * (dO.V^T - D), P and dS rounded to bf16 before the products, FP32 accumulation,
 * dQ = dS.K / 8, dK = dS^T.Q / 8, dV = P^T.dO.
 *
 *   q, k, v     [batch, heads, q_len | kv_len, 64] bf16 with element strides (same layout rules
 *               as tt_attn_forward_bf16; TT_ATTN_UNSUPPORTED otherwise)
 *   dout, out   contiguous [batch, heads, q_len, 64] bf16 (dO and the forward's O)
 *   lse         contiguous [batch, heads, q_len] FP32, natural log (the forward's LSE)
 *   dq          contiguous [batch, heads, q_len, 64] bf16 output
 *   dk, dv      contiguous [batch, heads, kv_len, 64] bf16 outputs
 *   workspace   tt_attn_backward_workspace_size() bytes, 16-byte aligned (the FP32 row sums D,
 *               the FP32 dQ accumulator and a work counter; its contents on entry do not matter)
 *
 * Mask: key j visible to query i iff j <= i + past_len, kv_len == q_len + past_len.
 * On `stream`, in order, three kernels: row sums D (which also zeroes the dQ accumulator and
 * the work counter), one persistent dQ/dK/dV kernel, dQ scaling to bf16. Nothing is allocated.
 */
TT_ATTN_API tt_attn_status tt_attn_backward_bf16(
    const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides, const void* dout, const void* out, const float* lse,
    int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int64_t head_dim,
    int64_t past_len, void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
    void* stream);

/*
 * Same contract as tt_attn_backward_bf16, with bit-identical results on every call: each output
 * element is accumulated by one CTA in a fixed order (three kernels: row sums D, a dQ kernel
 * over 128-row query tiles, a dK/dV kernel over 128-key tiles), where tt_attn_backward_bf16
 * adds the dQ contributions of different key tiles with reduce-adds in timing-dependent order.
 * The torch binding takes this path under torch.use_deterministic_algorithms(True); the
 * reference's own backward kernels use no atomics. Same workspace size.
 */
TT_ATTN_API tt_attn_status tt_attn_backward_bf16_deterministic(
    const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides, const void* dout, const void* out, const float* lse,
    int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int64_t head_dim,
    int64_t past_len, void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
    void* stream);

/* Bytes of workspace tt_attn_backward_bf16 needs (batch * heads * q_len FP32 row sums, padded
 * to 256 bytes, plus batch * heads * q_len * 64 FP32 for dQ), 0 for invalid sizes. */
TT_ATTN_API size_t tt_attn_backward_workspace_size(int64_t batch, int64_t heads, int64_t q_len);

/*
 * Fused rotary embedding + KV-cache append for one decoder layer (the step before attention
 * in Block.forward, tiny_transformer/model.py:61-68: reference.rope on q and k, reference.py:
 * 30-34, then KVCache.update, model.py:29-41). Replaces for this path the reference's
 * `rope` operator calls (student rope_forward) plus the two cache copies.
 *
 *   qkv      [batch, q_len, 3, heads, 64] bf16, contiguous (the fused QKV projection)
 *   cos, sin [table_len, 32] FP32 contiguous, row = position (rounded to bf16 as the
 *            reference's cos.to(x.dtype) does)
 *   q_out    [batch, heads, q_len, 64] bf16 contiguous: rope(q)
 *   cache_k / cache_v [batch, heads, capacity, 64] bf16, last stride 1, element strides in
 *            ck_strides / cv_strides (4 entries); row `position + t` receives rope(k) / v.
 *
 * The start position is `position` or, when `position_dev` is not NULL, the int64 it points
 * to on the device (read at run time, so a captured CUDA graph can serve every step). Host
 * positions are validated here (BAD_ARG); device-held ones by the kernel, which skips rows
 * outside [0, min(capacity, table_len)) and sets status bit 1. Bit-exact with the reference's
 * bf16 expression. All pointers 4-byte aligned; 16-byte aligned rows are fastest.
 */
TT_ATTN_API tt_attn_status tt_rope_append_bf16(
    const void* qkv, int64_t batch, int64_t q_len, int64_t heads, const float* cos,
    const float* sin, int64_t table_len, int64_t position, const int64_t* position_dev,
    void* q_out, void* cache_k, const int64_t* ck_strides, void* cache_v,
    const int64_t* cv_strides, int64_t capacity, void* stream);

/* QKV projection with RoPE and the KV-cache append in its epilogue, one kernel per layer: the
 * steps in front of the attention in the reference's Block.forward (model.py:59-67:
 * `linear(normalized, qkv)`, `rope(q)`, `rope(k)`, `KVCache.update`), with the projection never
 * written to memory.
 *   hidden   [batch * q_len, dim] bf16 row-major (the normalised hidden state), dim % 64 == 0
 *   w_qkv    [3 * heads * 64, dim] bf16 row-major (the layer's qkv weight)
 *   cos/sin  [table_len, 32] FP32 tables; position: first position (or position_dev, an int64
 *            on the device read at run time)
 *   q_out    [batch, heads, q_len, 64] bf16 contiguous = rope(q)
 *   cache_k/cache_v [batch, heads, capacity, 64] bf16 (unit last stride): rows position + t get
 *            rope(k) and v.
 * The projection is accumulated in FP32 and rounded to bf16, then rotated exactly as
 * tt_rope_append_bf16 rotates a bf16 projection. All pointers 16-byte aligned. The feature
 * tile width (16 to 128 features) is chosen per call so that the grid covers the SMs; the
 * result does not depend on it. */
TT_ATTN_API tt_attn_status tt_qkv_rope_append_bf16(
    const void* hidden, int64_t batch, int64_t q_len, int64_t dim, const void* w_qkv,
    int64_t heads, const float* cos, const float* sin, int64_t table_len, int64_t position,
    const int64_t* position_dev, void* q_out, void* cache_k, const int64_t* ck_strides,
    void* cache_v, const int64_t* cv_strides, int64_t capacity, void* stream);

/* Diagnostic for the failure path: launches one warp on `stream` that waits on a barrier
 * phase nothing completes, bounded by `budget_cycles` (1 .. 1e9 SM clock cycles). The wait
 * gives up by itself and sets bit 0 of the device status, which the caller then reads (and
 * clears) with tt_attn_device_status; the context stays usable. No counterpart in the
 * reference, which has no bounded waits. Returns BAD_ARG for a budget outside the range. */
TT_ATTN_API tt_attn_status tt_attn_selftest_wait_timeout(int64_t budget_cycles, void* stream);

/* Human-readable name of a status code. */
TT_ATTN_API const char* tt_attn_status_string(tt_attn_status status);

/* Message for the last non-OK status returned on the calling thread ("" if none). */
TT_ATTN_API const char* tt_attn_last_error(void);

TT_ATTN_API int tt_attn_abi_version(void);

/*
 * Single-token decode that allocates nothing, not even through the caller. No counterpart in
 * the reference: it exists for callers that cannot allocate device memory when they decode
 * (a server whose memory is entirely reserved by its own pools, a Go/Java/Rust host calling
 * this C ABI without a CUDA allocator, a loop that must stay out of the driver's allocator).
 *
 * Same computation and arguments as tt_attn_forward_bf16 with q_len = 1, head_dim = 64 and
 * past_len = kv_len - 1; the split-KV partials live in a static device array of 8 MiB
 * (8388608 bytes) that every GPU loading this library holds until exit. Shapes whose partials
 * exceed it (tt_attn_forward_workspace_size) return TT_ATTN_BAD_ARG; a device other than
 * sm_100 returns TT_ATTN_UNSUPPORTED. The first call on a device looks up the array's device
 * address (with that device current), and so does the first call after the current context
 * of that device changed (cudaDeviceReset, or a context the caller made current); make those
 * calls before any stream capture. All calls share the array: calls whose kernels overlap on
 * the GPU (different streams, or different host threads) race on it and must be serialised
 * by the caller. Caches of up to 2^20 (batch * heads * kv_len) K/V rows, or up to 2^21 in at
 * most 640 (batch, head) sequences, use no scratch at all.
 */
TT_ATTN_API tt_attn_status tt_attn_decode_bf16_noalloc(
    const void* q, const int64_t* q_strides,
    const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides,
    int64_t batch, int64_t heads, int64_t kv_len, const int32_t* kv_lens,
    void* out, float* lse, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TT_ATTENTION_H_ */
