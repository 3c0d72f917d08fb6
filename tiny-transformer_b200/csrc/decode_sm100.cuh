// Single-token (Tq == 1) KV-cache decode for sm_100a: split-KV with an FP32 LSE combine.
//
// Semantics follow the reference decode path (Tiny-transformer
// csrc/attention/attention_decode_BF16_kernel.cuh:45-128 and reference.py:49-53): the query
// attends to every cached key (Tk == past_len + 1), scale 1/sqrt(64), FP32 softmax, BF16 O,
// natural-log FP32 LSE. Added here: an optional per-sequence valid length kv_lens[b]
// (key j visible iff j < kv_lens[b]); a sequence with no visible key gets O = 0, LSE = -inf,
// the reference's convention for rows without visible keys.
//
// Decode is HBM-bound, so the kernel is built around moving K/V rows at full bandwidth:
// one CTA owns `chunk` keys of one (batch, head); a single thread issues 1-D bulk async
// copies (TMA engine, no multicast) of the whole chunk into shared memory, one mbarrier per
// 64-row sub-tile, so the copy of later sub-tiles overlaps compute on earlier ones. Rows are
// read through the cache strides, so prefix views of a larger cache need no copy.
// Compute: 16 lane-groups of 8 lanes; a group owns one key row at a time (16 B per lane),
// dot products reduce with 3 xor-shuffles, each group keeps an online softmax (m, l, acc),
// and the groups merge through shared memory at the end.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace tt {
namespace decode {

constexpr int HD = 64;
constexpr int ROW_BYTES = HD * 2;           // 128 B per key row
constexpr int SUB = 64;                     // rows per sub-tile / mbarrier
constexpr int MAX_SUBS = 4;                 // chunk <= 256 rows
constexpr int MAX_CHUNK = SUB * MAX_SUBS;
constexpr int THREADS = 128;
constexpr int GROUPS = THREADS / 8;         // 16 lane-groups
constexpr int PARTIAL = HD + 2;             // acc[64], m (log2 units), l
constexpr float LN2 = 0.69314718055994530942f;

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_sb, q_sh;          // element strides of q [B,H,1,64]
  int64_t k_sb, k_sh, k_st;    // element strides of k [B,H,Tk,64]
  int64_t v_sb, v_sh, v_st;
  const int32_t* kv_lens;      // optional [B]
  int B, H;
  int Tk;
  int chunk;                   // keys per CTA, multiple of SUB, <= MAX_CHUNK
  int n_chunks;                // ceil(Tk / chunk)
  __nv_bfloat16* o;            // contiguous [B,H,1,64]
  float* lse;                  // [B,H,1]
  float* partials;             // [B*H, n_chunks, PARTIAL] (used when n_chunks > 1)
  float scale_log2;
};

__device__ __forceinline__ int valid_len(const Params& p, int b) {
  if (p.kv_lens == nullptr) return p.Tk;
  const int L = p.kv_lens[b];
  return L < 0 ? 0 : (L > p.Tk ? p.Tk : L);
}

__device__ __forceinline__ int chunks_for(int L, int chunk) {
  return L <= 0 ? 1 : (L + chunk - 1) / chunk;
}

__device__ __forceinline__ void load_row8(const uint8_t* src, float (&f)[8]) {
  const uint4 u = *reinterpret_cast<const uint4*>(src);
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x);
  f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z);
  f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}

__global__ void __launch_bounds__(THREADS)
decode_split_kernel(const Params p) {
  extern __shared__ __align__(128) uint8_t smem[];  // K rows then V rows, chunk x 128 B each
  __shared__ uint64_t bars[MAX_SUBS];
  __shared__ float red_m[GROUPS];
  __shared__ float red_l[GROUPS];
  __shared__ float red_acc[GROUPS][HD];

  const int tid = threadIdx.x;
  const long long cta = blockIdx.x;
  const int bh = static_cast<int>(cta / p.n_chunks);
  const int c = static_cast<int>(cta % p.n_chunks);
  const int b = bh / p.H;
  const int h = bh % p.H;
  const int L = valid_len(p, b);
  const int nc = chunks_for(L, p.chunk);
  if (c >= nc) return;
  const int start = c * p.chunk;
  const int rows = max(0, min(p.chunk, L - start));
  const int nsub = (rows + SUB - 1) / SUB;
  uint8_t* ks = smem;
  uint8_t* vs = smem + static_cast<size_t>(p.chunk) * ROW_BYTES;

  if (tid == 0) {
    for (int i = 0; i < nsub; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  __syncthreads();

  const __nv_bfloat16* kb = p.k + b * p.k_sb + h * p.k_sh + static_cast<int64_t>(start) * p.k_st;
  const __nv_bfloat16* vb = p.v + b * p.v_sb + h * p.v_sh + static_cast<int64_t>(start) * p.v_st;
  if (tid < 32) {
    const uint64_t pol = l2_policy_evict_first();
    if (tid == 0) {
      for (int i = 0; i < nsub; ++i) {
        const int r = min(SUB, rows - i * SUB);
        mbar_arrive_expect_tx(&bars[i], static_cast<uint32_t>(2 * r * ROW_BYTES));
      }
    }
    __syncwarp();
    if (p.k_st == HD && p.v_st == HD) {
      // Rows are contiguous: one copy per sub-tile for K and one for V.
      if (tid == 0) {
        for (int i = 0; i < nsub; ++i) {
          const int r = min(SUB, rows - i * SUB);
          bulk_load(ks + i * SUB * ROW_BYTES, kb + static_cast<int64_t>(i) * SUB * HD,
                    r * ROW_BYTES, &bars[i], pol);
          bulk_load(vs + i * SUB * ROW_BYTES, vb + static_cast<int64_t>(i) * SUB * HD,
                    r * ROW_BYTES, &bars[i], pol);
        }
      }
    } else {
      // Strided rows (16-byte aligned): one 128-byte copy per row, spread over the warp.
      for (int r = tid; r < rows; r += 32) {
        bulk_load(ks + r * ROW_BYTES, kb + r * p.k_st, ROW_BYTES, &bars[r / SUB], pol);
        bulk_load(vs + r * ROW_BYTES, vb + r * p.v_st, ROW_BYTES, &bars[r / SUB], pol);
      }
    }
  }

  // q: lane j of a group holds features [8j, 8j+8), pre-multiplied by scale*log2(e).
  const int g = tid >> 3;
  const int j = tid & 7;
  float qf[8];
  {
    const uint8_t* qrow = reinterpret_cast<const uint8_t*>(p.q + b * p.q_sb + h * p.q_sh);
    load_row8(qrow + j * 16, qf);
#pragma unroll
    for (int i = 0; i < 8; ++i) qf[i] *= p.scale_log2;
  }

  float m = -INFINITY, l = 0.f;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.f;
  bool ok = true;

  for (int sidx = 0; sidx < nsub; ++sidx) {
    if (!__all_sync(0xffffffffu, mbar_wait(&bars[sidx], 0))) { ok = false; break; }
    const int r_end = min(rows, (sidx + 1) * SUB);
    // Each group handles rows sidx*SUB + g + 16*i, i = 0..3, as one batch.
    float x[SUB / GROUPS];
#pragma unroll
    for (int i = 0; i < SUB / GROUPS; ++i) {
      const int r = sidx * SUB + g + GROUPS * i;
      float kf[8];
      float d = 0.f;
      if (r < r_end) {
        load_row8(ks + r * ROW_BYTES + j * 16, kf);
#pragma unroll
        for (int t = 0; t < 8; ++t) d = fmaf(qf[t], kf[t], d);
      }
      d += __shfl_xor_sync(0xffffffffu, d, 1);
      d += __shfl_xor_sync(0xffffffffu, d, 2);
      d += __shfl_xor_sync(0xffffffffu, d, 4);
      x[i] = r < r_end ? d : -INFINITY;
    }
    float mx = x[0];
#pragma unroll
    for (int i = 1; i < SUB / GROUPS; ++i) mx = fmaxf(mx, x[i]);
    const float m_new = fmaxf(m, mx);
    if (m_new == -INFINITY) continue;  // no valid row for this group in this sub-tile
    const float f = ex2_approx(m - m_new);  // m == -inf -> 0
    l *= f;
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] *= f;
#pragma unroll
    for (int i = 0; i < SUB / GROUPS; ++i) {
      const int r = sidx * SUB + g + GROUPS * i;
      if (r < r_end) {
        const float pr = ex2_approx(x[i] - m_new);
        l += pr;
        float vf[8];
        load_row8(vs + r * ROW_BYTES + j * 16, vf);
#pragma unroll
        for (int t = 0; t < 8; ++t) acc[t] = fmaf(pr, vf[t], acc[t]);
      }
    }
    m = m_new;
  }
  ok = __syncthreads_and(ok);

  if (ok) {
    if (j == 0) {
      red_m[g] = m;
      red_l[g] = l;
    }
#pragma unroll
    for (int t = 0; t < 8; ++t) red_acc[g][j * 8 + t] = acc[t];
  }
  __syncthreads();
  if (!ok) {
    // Drain: do not retire the CTA while a bulk copy into its shared memory is pending.
    if (tid == 0)
      for (int i = 0; i < nsub; ++i) mbar_wait(&bars[i], 0);
    return;
  }

  if (tid < HD) {
    float M = -INFINITY;
#pragma unroll
    for (int i = 0; i < GROUPS; ++i) M = fmaxf(M, red_m[i]);
    float num = 0.f, den = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int i = 0; i < GROUPS; ++i) {
        if (red_m[i] == -INFINITY) continue;
        const float w = ex2_approx(red_m[i] - M);
        num = fmaf(w, red_acc[i][tid], num);
        den = fmaf(w, red_l[i], den);
      }
    }
    if (nc == 1) {
      const float out = den > 0.f ? num / den : 0.f;
      p.o[static_cast<size_t>(bh) * HD + tid] = __float2bfloat16_rn(out);
      if (tid == 0) p.lse[bh] = den > 0.f ? (M + log2f(den)) * LN2 : -INFINITY;
    } else {
      float* dst = p.partials + (static_cast<size_t>(bh) * p.n_chunks + c) * PARTIAL;
      dst[tid] = num;
      if (tid == 0) {
        dst[HD] = M;
        dst[HD + 1] = den;
      }
    }
  }
}

// Merge the per-chunk partials of one (batch, head): rescale numerators and denominators
// by exp2(m_c - M) before summing (never average normalised outputs).
__global__ void __launch_bounds__(HD)
decode_combine_kernel(const Params p) {
  const int bh = blockIdx.x;
  const int d = threadIdx.x;
  const int b = bh / p.H;
  const int L = valid_len(p, b);
  const int nc = chunks_for(L, p.chunk);
  if (nc <= 1) return;  // written directly by the split kernel
  const float* src = p.partials + static_cast<size_t>(bh) * p.n_chunks * PARTIAL;
  float M = -INFINITY;
  for (int c = 0; c < nc; ++c) M = fmaxf(M, src[c * PARTIAL + HD]);
  float num = 0.f, den = 0.f;
  if (M != -INFINITY) {
    for (int c = 0; c < nc; ++c) {
      const float mc = src[c * PARTIAL + HD];
      if (mc == -INFINITY) continue;
      const float w = ex2_approx(mc - M);
      num = fmaf(w, src[c * PARTIAL + d], num);
      den = fmaf(w, src[c * PARTIAL + HD + 1], den);
    }
  }
  const float out = den > 0.f ? num / den : 0.f;
  p.o[static_cast<size_t>(bh) * HD + d] = __float2bfloat16_rn(out);
  if (d == 0) p.lse[bh] = den > 0.f ? (M + log2f(den)) * LN2 : -INFINITY;
}

}  // namespace decode
}  // namespace tt
