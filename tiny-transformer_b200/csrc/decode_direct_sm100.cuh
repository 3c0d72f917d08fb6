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
// the cluster takes keys [r * keys_per_cta, (r + 1) * keys_per_cta) in chunks of 128 keys.
// Thread 0 loads each chunk's K and V rows with 4-D TMA tensor maps over [B, H, Tk, 64]
// (128-byte swizzle: 16-byte piece c of row r lands at piece c ^ (r % 8); no multicast) into a
// two-stage ring on mbarriers, so a CTA's next chunk streams in while the current one is
// reduced. Each of the 4 warps takes 32 keys of a chunk. Scores: lane i owns key i, holds q
// (pre-scaled FP32) in registers and reads its K row's eight pieces in swizzled order, which
// spreads a warp's 16-byte reads over all banks. P.V: lane i owns output features 2i, 2i + 1
// and reads that pair of each of the warp's 32 V rows (one 128-byte row per instruction),
// while p_r is broadcast by shuffle. (Per-lane global loads of the rows held a 128-key pass at
// ~3.5 us on L2-resident caches; a lane-per-feature score layout needed a 31-shuffle butterfly
// per 32 keys.) Warps keep an online softmax across chunks; the CTA merges its warps in shared
// memory. A sequence on one CTA writes O and LSE from there, with no cluster barrier (a
// barrier.cluster costs ~0.7 us even for a cluster of one). Otherwise every CTA writes its
// (m, l, acc) record into the cluster leader's shared memory (st.shared::cluster), one cluster
// barrier (release / acquire) publishes them, and the leader merges the records into O and
// LSE (per-CTA mbarrier arrivals on the leader measured ~1 us slower than the barrier). All CTAs
// of a cluster are co-scheduled and every CTA reaches the barrier exactly once (a timed-out wait
// skips the remaining chunks, after the copies in flight have landed), so the barrier always
// completes. Two 32 KiB stages per CTA
// leave room for three CTAs per SM; the host sizes the split so that the grid fills them.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace tt {
namespace decode_direct {

constexpr int HD = 64;
constexpr int WARPS = 4;
constexpr int THREADS = WARPS * 32;
constexpr int KEYS_PER_PASS = THREADS;  // keys per chunk: 32 per warp
constexpr int STAGES = 2;
constexpr uint32_t ROW_BYTES = HD * 2;
constexpr uint32_t CHUNK_BYTES = KEYS_PER_PASS * ROW_BYTES;  // 16 KiB of K (and of V)
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

struct alignas(1024) Smem {
  uint8_t k[STAGES][CHUNK_BYTES];
  uint8_t v[STAGES][CHUNK_BYTES];
  float rec[WARPS][REC];       // this CTA's warps
  float crec[MAX_SPLITS][REC];  // the cluster's CTAs (leader only)
  uint64_t full[STAGES], empty[STAGES];
  volatile int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack for 1 KiB alignment (swizzle)

__device__ __forceinline__ void unpack8(const uint4 u, float (&f)[8]) {
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x);
  f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z);
  f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}

// Bounded wait that gives up as soon as another warp of the CTA has given up.
__device__ __forceinline__ bool wait_or_abort(Smem& s, uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (s.abort) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      atomicOr(&g_tt_status, TT_ERR_TIMEOUT);
      s.abort = 1;
      return false;
    }
  }
}

__global__ void __launch_bounds__(THREADS, 3)
decode_direct_kernel(const __grid_constant__ CUtensorMap tm_k,
                     const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int rank = static_cast<int>(cluster_ctarank());
  const int bh = static_cast<int>(blockIdx.x) / p.splits;
  const int b = bh / p.H, h = bh - b * p.H;
  // q (every lane reads the whole row: broadcasts) and the sequence length are requested first.
  uint4 qraw[8];
  {
    const uint4* qrow = reinterpret_cast<const uint4*>(p.q + b * p.q_sb + h * p.q_sh);
#pragma unroll
    for (int c = 0; c < 8; ++c) qraw[c] = __ldg(qrow + c);
  }
  int L = p.Tk;
  if (p.kv_lens != nullptr) L = min(max(__ldg(p.kv_lens + b), 0), p.Tk);
  const int k_begin = rank * p.keys_per_cta;
  const int k_end = min(L, k_begin + p.keys_per_cta);
  const int n_chunks = k_end > k_begin ? (k_end - k_begin + KEYS_PER_PASS - 1) / KEYS_PER_PASS : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], WARPS);
    }
    s.abort = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  __syncthreads();

  // Chunk c into stage c % STAGES: the 128 rows from k_begin + 128 c (rows past Tk read as
  // zero; rows past k_end are loaded and never used). Thread 0 only.
  auto issue_chunk = [&](int c) {
    const int st = c % STAGES;
    const int row0 = k_begin + c * KEYS_PER_PASS;
    mbar_arrive_expect_tx(&s.full[st], 2 * CHUNK_BYTES);
    tma_load_4d(s.k[st], &tm_k, &s.full[st], 0, row0, h, b);
    tma_load_4d(s.v[st], &tm_v, &s.full[st], 0, row0, h, b);
  };
  if (threadIdx.x == 0)
    for (int c = 0; c < min(STAGES, n_chunks); ++c) issue_chunk(c);

  // q * scale * log2(e) in FP32 registers.
  float qv[HD];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    float f[8];
    unpack8(qraw[c], f);
#pragma unroll
    for (int i = 0; i < 8; ++i) qv[8 * c + i] = f[i] * p.scale_log2;
  }
  int issued = min(STAGES, n_chunks);

  float m = -INFINITY;       // warp-uniform running max (log2 units)
  float l = 0.f;             // this lane's share of the running sum
  float a0 = 0.f, a1 = 0.f;  // output features 2*lane, 2*lane + 1
  for (int c = 0; c < n_chunks; ++c) {
    const int st = c % STAGES;
    if (!__all_sync(0xffffffffu, wait_or_abort(s, &s.full[st], (c / STAGES) & 1))) break;
    const int n_valid = min(32, k_end - (k_begin + c * KEYS_PER_PASS) - warp * 32);  // uniform
    if (n_valid > 0) {
      const uint32_t kbase = smem_u32(s.k[st]) + warp * 32 * ROW_BYTES;
      const uint32_t vbase = smem_u32(s.v[st]) + warp * 32 * ROW_BYTES;
      // Score of key `lane` of this warp: its row's pieces in swizzled order.
      const uint32_t krow = kbase + lane * ROW_BYTES;
      const uint32_t ksw = static_cast<uint32_t>(lane & 7);
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float kf[8];
        unpack8(lds_u4(krow + ((static_cast<uint32_t>(c) ^ ksw) << 4)), kf);
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i & 3] = fmaf(qv[8 * c + i], kf[i], d[i & 3]);
      }
      const float x = lane < n_valid ? (d[0] + d[1]) + (d[2] + d[3]) : -INFINITY;
      float mx = x;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m, mx);  // finite: the chunk has at least one valid row here
      const float f = ex2_approx(m - m_new);   // m == -inf -> 0
      const float pr = ex2_approx(x - m_new);  // rows past the range: exp2(-inf) = 0
      l = l * f + pr;
      float b0[4] = {a0 * f, 0.f, 0.f, 0.f}, b1[4] = {a1 * f, 0.f, 0.f, 0.f};
      // Features 2 lane, 2 lane + 1 of V row rr: byte 4 lane of the row, in piece lane / 4.
      // Per half of the rows, all shared loads first, then all broadcasts of p, then the
      // products: interleaved, each row's load waited for the previous row's shuffle and the
      // loop ran as one latency chain (~1.7 us per chunk).
      const uint32_t vcol = static_cast<uint32_t>(lane & 3) << 2;
      const uint32_t vpiece = static_cast<uint32_t>(lane >> 2);
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t vv[16];
        float pb[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int rr = half * 16 + i;
          vv[i] = rr < n_valid ? lds_u32(vbase + rr * ROW_BYTES +
                                         ((vpiece ^ static_cast<uint32_t>(rr & 7)) << 4) + vcol)
                               : 0u;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) pb[i] = __shfl_sync(0xffffffffu, pr, half * 16 + i);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          b0[i & 3] = fmaf(pb[i], bf16_lo(vv[i]), b0[i & 3]);
          b1[i & 3] = fmaf(pb[i], bf16_hi(vv[i]), b1[i & 3]);
        }
      }
      a0 = (b0[0] + b0[1]) + (b0[2] + b0[3]);
      a1 = (b1[0] + b1[1]) + (b1[2] + b1[3]);
      m = m_new;
    }
    // This warp is done with the stage; warp 0 refills it once every warp is.
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.empty[st]);
    if (warp == 0 && issued < n_chunks) {
      if (!__all_sync(0xffffffffu, wait_or_abort(s, &s.empty[st], (c / STAGES) & 1))) break;
      if (lane == 0) issue_chunk(issued);
      ++issued;
    }
  }
  if (threadIdx.x == 0 && s.abort) {
    // Never leave while a TMA write into this CTA's shared memory is pending.
    for (int c = max(0, issued - STAGES); c < issued; ++c)
      mbar_wait(&s.full[c % STAGES], (c / STAGES) & 1);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
  reinterpret_cast<float2*>(s.rec[warp])[lane] = make_float2(a0, a1);
  if (lane == 0) {
    s.rec[warp][HD] = m;
    s.rec[warp][HD + 1] = l;
  }
  __syncthreads();
  // Warp 0 merges the CTA's warps (weights exp2(m_w - M), never averaged outputs): the output
  // of a sequence on one CTA, else the CTA's record for the leader's crec[rank].
  float M = -INFINITY, n0 = 0.f, n1 = 0.f, den = 0.f;
  if (warp == 0) {
#pragma unroll
    for (int w = 0; w < WARPS; ++w) M = fmaxf(M, s.rec[w][HD]);
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < WARPS; ++w) {
        const float mw = s.rec[w][HD];
        if (mw == -INFINITY) continue;
        const float wt = ex2_approx(mw - M);
        const float2 a = reinterpret_cast<const float2*>(s.rec[w])[lane];
        n0 = fmaf(wt, a.x, n0);
        n1 = fmaf(wt, a.y, n1);
        den = fmaf(wt, s.rec[w][HD + 1], den);
      }
    }
    if (p.splits > 1) {
      const uint32_t dst = map_to_rank(smem_u32(s.crec[rank]), 0);
      st_cluster_f32x2(dst + lane * 8, n0, n1);
      if (lane == 0) {
        st_cluster_f32(dst + HD * 4, M);
        st_cluster_f32(dst + (HD + 1) * 4, den);
      }
    }
  }
  if (p.splits > 1) {
    cluster_sync();
    if (rank != 0 || warp != 0) return;
    M = -INFINITY;
    for (int c = 0; c < p.splits; ++c) M = fmaxf(M, s.crec[c][HD]);
    n0 = n1 = den = 0.f;
    if (M != -INFINITY) {
      for (int c = 0; c < p.splits; ++c) {
        const float mc = s.crec[c][HD];
        if (mc == -INFINITY) continue;
        const float wt = ex2_approx(mc - M);
        const float2 a = reinterpret_cast<const float2*>(s.crec[c])[lane];
        n0 = fmaf(wt, a.x, n0);
        n1 = fmaf(wt, a.y, n1);
        den = fmaf(wt, s.crec[c][HD + 1], den);
      }
    }
  } else if (warp != 0) {
    return;
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  reinterpret_cast<uint32_t*>(p.o + static_cast<size_t>(bh) * HD)[lane] =
      pack_bf16x2(n0 * inv, n1 * inv);
  if (lane == 0) p.lse[bh] = den > 0.f ? (M + log2f(den)) * LN2 : -INFINITY;
}

}  // namespace decode_direct
}  // namespace tt
