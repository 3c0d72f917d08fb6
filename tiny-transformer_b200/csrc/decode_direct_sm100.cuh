// Single-token decode of short and medium KV caches for sm_100a: each sequence's keys are
// split over the CTAs of one thread-block cluster, whose partial softmax results merge through
// distributed shared memory. No workspace, no memset, one launch.
//
// Same semantics as decode_sm100.cuh (Tiny-transformer csrc/attention/
// attention_decode_BF16_kernel.cuh:45-128 and reference.py:49-53): the query attends to every
// cached key, or to the first kv_lens[b] when lengths are given; FP32 softmax; BF16 O;
// natural-log FP32 LSE; O = 0 and LSE = -inf for a sequence without visible keys.
//
// The persistent split-KV kernel pays a fixed cost per call (a counter memset, 148 CTAs that
// set up a bulk-copy ring, 384-key stages, a cross-CTA merge through global memory) that
// dominates below a few hundred MB of cache. Here a (batch, head) sequence is one cluster of
// `splits` CTAs (grid.x = splits * B * H, cluster dims (splits, 1, 1), splits <= 8); CTA r of
// the cluster takes keys [r * keys_per_cta, (r + 1) * keys_per_cta) in passes of 128 keys.
// Each of the 4 warps takes 32 keys per pass, one key row per lane: the lane loads its K row
// (eight 16-byte loads of one 128-byte line) and forms the dot product with q (FP32,
// pre-scaled, read from shared memory as broadcasts); the warp takes the max, each lane its
// exponential, and for P.V each lane owns two output features and reads row r's pair of V
// values (the warp reads the row's 128 bytes together) while p_r is broadcast by shuffle. The
// V loads of a pass are issued before the scores are reduced. Warps keep an online softmax
// across passes; the CTA merges its warps in shared memory, every CTA writes its (m, l, acc)
// record into the cluster leader's shared memory (st.shared::cluster), one cluster barrier
// (release / acquire) publishes them, and the leader merges the records into O and LSE.
// All CTAs of a cluster are co-scheduled and every CTA reaches the barrier exactly once, so
// the barrier always completes. 128 registers per thread (no spills) keep 4 CTAs per SM.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace tt {
namespace decode_direct {

constexpr int HD = 64;
constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int KEYS_PER_PASS = THREADS;  // one key row per thread
constexpr int MAX_SPLITS = 8;           // portable cluster size
constexpr int REC = HD + 2;             // acc[64], m (log2 units), l
constexpr float LN2 = 0.69314718055994530942f;

struct Params {
  const __nv_bfloat16* q;
  const __nv_bfloat16* k;
  const __nv_bfloat16* v;
  int64_t q_sb, q_sh;        // element strides of q [B,H,1,64]
  int64_t k_sb, k_sh, k_st;  // element strides of k [B,H,Tk,64]
  int64_t v_sb, v_sh, v_st;
  const int32_t* kv_lens;    // optional [B]
  int B, H, Tk;
  int splits;                // CTAs per sequence = cluster size
  int keys_per_cta;          // multiple of KEYS_PER_PASS
  __nv_bfloat16* o;          // contiguous [B,H,1,64]
  float* lse;                // [B,H,1]
  float scale_log2;
};

__device__ __forceinline__ void unpack8(const uint4 u, float (&f)[8]) {
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x);
  f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z);
  f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}

__global__ void __launch_bounds__(THREADS, 4)
decode_direct_kernel(const Params p) {
  __shared__ __align__(16) float qs[HD];
  __shared__ __align__(16) float rec[WARPS][REC];       // this CTA's warps
  __shared__ __align__(16) float crec[MAX_SPLITS][REC];  // the cluster's CTAs (leader only)
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int bh = static_cast<int>(blockIdx.x) / p.splits;
  const int b = bh / p.H, h = bh - b * p.H;
  // The q pair this thread stages (threads 0-31) and the sequence length are requested first;
  // the first pass's K and V rows are requested before q is staged in shared memory, so the
  // q round trip overlaps the K/V one.
  uint32_t qpair = 0;
  if (threadIdx.x < HD / 2)
    qpair = __ldg(reinterpret_cast<const uint32_t*>(p.q + b * p.q_sb + h * p.q_sh) + threadIdx.x);
  int L = p.Tk;
  if (p.kv_lens != nullptr) L = min(max(__ldg(p.kv_lens + b), 0), p.Tk);
  const int k_begin = rank * p.keys_per_cta;
  const int k_end = min(L, k_begin + p.keys_per_cta);
  const __nv_bfloat16* kb = p.k + b * p.k_sb + h * p.k_sh;
  const __nv_bfloat16* vb = p.v + b * p.v_sb + h * p.v_sh;
  // Row stride of V in bf16 pairs (strides are multiples of 8 elements; a row step fits int).
  const int v_pairs = static_cast<int>(p.v_st >> 1);

  // Requests of one pass: this lane's K row and the pass's V row pairs (rows below n_valid).
  auto load_pass = [&](int base, int n_valid, uint4 (&kr)[8], uint32_t (&vv)[32]) {
    if (lane < n_valid) {
      const uint4* krow =
          reinterpret_cast<const uint4*>(kb + static_cast<int64_t>(base + lane) * p.k_st);
#pragma unroll
      for (int c = 0; c < 8; ++c) kr[c] = __ldg(krow + c);
    }
    const uint32_t* vrow =
        reinterpret_cast<const uint32_t*>(vb + static_cast<int64_t>(base) * p.v_st) + lane;
#pragma unroll
    for (int rr = 0; rr < 32; ++rr)
      if (rr < n_valid) vv[rr] = __ldg(vrow + rr * v_pairs);
  };

  uint4 kr[8];
  uint32_t vv[32];
  int base = k_begin + warp * 32;
  if (base < k_end) load_pass(base, min(32, k_end - base), kr, vv);

  // q * scale * log2(e) in shared memory (FP32); every lane reads it as broadcasts.
  if (threadIdx.x < HD / 2) {
    qs[2 * threadIdx.x] = bf16_lo(qpair) * p.scale_log2;
    qs[2 * threadIdx.x + 1] = bf16_hi(qpair) * p.scale_log2;
  }
  __syncthreads();
  const uint32_t qaddr = smem_u32(qs);

  float m = -INFINITY;       // warp-uniform running max (log2 units)
  float l = 0.f;             // this lane's share of the running sum
  float a0 = 0.f, a1 = 0.f;  // output features 2*lane, 2*lane + 1
  for (; base < k_end; base += KEYS_PER_PASS) {
    const int n_valid = min(32, k_end - base);  // warp-uniform
    if (base != k_begin + warp * 32) load_pass(base, n_valid, kr, vv);
    float x = -INFINITY;
    if (lane < n_valid) {
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float kf[8];
        unpack8(kr[c], kf);
        const float4 qa = lds_f4(qaddr + c * 32), qb = lds_f4(qaddr + c * 32 + 16);
        d[0] = fmaf(qa.x, kf[0], d[0]);
        d[1] = fmaf(qa.y, kf[1], d[1]);
        d[2] = fmaf(qa.z, kf[2], d[2]);
        d[3] = fmaf(qa.w, kf[3], d[3]);
        d[0] = fmaf(qb.x, kf[4], d[0]);
        d[1] = fmaf(qb.y, kf[5], d[1]);
        d[2] = fmaf(qb.z, kf[6], d[2]);
        d[3] = fmaf(qb.w, kf[7], d[3]);
      }
      x = (d[0] + d[1]) + (d[2] + d[3]);
    }
    float mx = x;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m, mx);  // finite: the pass has at least one valid row
    const float f = ex2_approx(m - m_new);   // m == -inf -> 0
    const float pr = ex2_approx(x - m_new);  // rows past the range: exp2(-inf) = 0
    l = l * f + pr;
    float b0[4] = {a0 * f, 0.f, 0.f, 0.f}, b1[4] = {a1 * f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int rr = 0; rr < 32; ++rr) {
      if (rr < n_valid) {
        const float pb = __shfl_sync(0xffffffffu, pr, rr);
        b0[rr & 3] = fmaf(pb, bf16_lo(vv[rr]), b0[rr & 3]);
        b1[rr & 3] = fmaf(pb, bf16_hi(vv[rr]), b1[rr & 3]);
      }
    }
    a0 = (b0[0] + b0[1]) + (b0[2] + b0[3]);
    a1 = (b1[0] + b1[1]) + (b1[2] + b1[3]);
    m = m_new;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
  reinterpret_cast<float2*>(rec[warp])[lane] = make_float2(a0, a1);
  if (lane == 0) {
    rec[warp][HD] = m;
    rec[warp][HD + 1] = l;
  }
  __syncthreads();
  // Warp 0 merges the CTA's warps (weights exp2(m_w - M), never averaged outputs) and writes
  // the CTA's record into the leader's crec[rank].
  if (warp == 0) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, rec[w][HD]);
    float n0 = 0.f, n1 = 0.f, den = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        const float mw = rec[w][HD];
        if (mw == -INFINITY) continue;
        const float wt = ex2_approx(mw - M);
        const float2 a = reinterpret_cast<const float2*>(rec[w])[lane];
        n0 = fmaf(wt, a.x, n0);
        n1 = fmaf(wt, a.y, n1);
        den = fmaf(wt, rec[w][HD + 1], den);
      }
    }
    const uint32_t dst = map_to_rank(smem_u32(crec[rank]), 0);
    st_cluster_f32x2(dst + lane * 8, n0, n1);
    if (lane == 0) {
      st_cluster_f32(dst + HD * 4, M);
      st_cluster_f32(dst + (HD + 1) * 4, den);
    }
  }
  cluster_sync();
  if (rank != 0 || warp != 0) return;
  float M = -INFINITY;
  for (int c = 0; c < p.splits; ++c) M = fmaxf(M, crec[c][HD]);
  float n0 = 0.f, n1 = 0.f, den = 0.f;
  if (M != -INFINITY) {
    for (int c = 0; c < p.splits; ++c) {
      const float mc = crec[c][HD];
      if (mc == -INFINITY) continue;
      const float wt = ex2_approx(mc - M);
      const float2 a = reinterpret_cast<const float2*>(crec[c])[lane];
      n0 = fmaf(wt, a.x, n0);
      n1 = fmaf(wt, a.y, n1);
      den = fmaf(wt, crec[c][HD + 1], den);
    }
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  reinterpret_cast<uint32_t*>(p.o + static_cast<size_t>(bh) * HD)[lane] =
      pack_bf16x2(n0 * inv, n1 * inv);
  if (lane == 0) p.lse[bh] = den > 0.f ? (M + log2f(den)) * LN2 : -INFINITY;
}

}  // namespace decode_direct
}  // namespace tt
