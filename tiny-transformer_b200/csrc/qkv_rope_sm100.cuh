// QKV projection with RoPE and the KV-cache append in its epilogue, for one decoder layer (the
// steps in front of the attention in Tiny-transformer's Block.forward, model.py:59-67):
//
//   qkv[m, n] = bf16( sum_k h[m, k] * W[n, k] )          (F.linear: FP32 accumulation, bf16 out)
//   q_out[b, h, t]            = rope(q part of row m = b * T + t)
//   cache_k[b, h, pos + t]    = rope(k part),  cache_v[b, h, pos + t] = v part
//
// with h the normalised hidden state [M = B * T, K] and W the layer's qkv weight [3 * H * 64, K]
// (both row-major, bf16). RoPE is applied to the bf16-rounded projection exactly as
// rope_append_sm100.cuh does it (reference.py:30-34 operation by operation in bf16), so the
// fused kernel's output equals rope_append applied to this kernel's own projection; against a
// projection computed by another GEMM (cuBLAS) it can differ by the rounding of FP32 sums
// accumulated in another order (one bf16 ulp, rarely).
//
// One CTA computes a 128-row x BN-feature tile of one of q, k, v: a TMA producer warp streams
// 64-wide K slices of h and W through a STAGES-deep ring (128-byte swizzle, no multicast), one
// thread issues tcgen05.mma (M = 128, N = BN, both operands K-major) into a TMEM accumulator,
// and four epilogue warps (thread = token row = TMEM lane) read the accumulator, round, rotate
// and store each head's row segment. The feature tile width BN (16, 32, 64 or 128) is chosen
// per call so that the grid fills the SMs: a decode step has one row tile (B * T <= 128 rows),
// and 128-feature tiles would leave most SMs idle while each CTA walks the whole K range. With
// a single row tile the h box is only as tall as the rows that exist (rounded up to 8); the
// MMA still reads 128 rows of A, and the accumulator rows beyond the box, computed from stale
// shared memory, are never stored. Rows past M are not stored. A device-held start position
// outside the cache or the table skips the row and sets TT_ERR_RANGE, as rope_append does.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace tt {
namespace qkv_rope {

constexpr int HD = 64;
constexpr int BM = 128;     // token rows per tile (the MMA's M)
constexpr int BK = 64;      // K slice per stage (128 bytes of bf16)
constexpr int PRODUCER_WARP = 0, MMA_WARP = 1, EPI_WARP0 = 2;
constexpr int THREADS = 6 * 32;
constexpr uint32_t A_SLICE_BYTES = BM * BK * 2;  // 16 KiB: the MMA reads all 128 rows

// Per feature-tile width: ring depth (about 200 KiB of stages), TMEM columns (at least 32) and
// the accumulator columns one tcgen05.ld brings in (one head segment of the epilogue).
template <int BN>
struct Tile {
  static_assert(BN == 16 || BN == 32 || BN == 64 || BN == 128, "feature tile width");
  static constexpr int STAGES = BN == 128 ? 6 : BN == 64 ? 8 : BN == 32 ? 10 : 12;
  static constexpr uint32_t B_SLICE_BYTES = BN * BK * 2;
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  static constexpr int SEG = BN < 32 ? BN : 32;
};

struct Params {
  int M, T, H, K;                 // M = B * T rows, H heads, K input features
  uint32_t stage_tx_bytes;        // bytes one stage's two TMA boxes deliver
  const float* cos;               // [table_len, 32]
  const float* sin;
  long long table_len;
  long long position;             // start position when position_dev is null
  const long long* position_dev;  // optional device-held start position
  __nv_bfloat16* q_out;           // contiguous [B, H, T, 64]
  __nv_bfloat16* cache_k;
  __nv_bfloat16* cache_v;
  long long ck_s0, ck_s1, ck_s2;  // element strides of cache_k (batch, head, position)
  long long cv_s0, cv_s1, cv_s2;
  long long capacity;
};

template <int BN>
struct alignas(1024) Smem {
  uint8_t a[Tile<BN>::STAGES][A_SLICE_BYTES];
  uint8_t b[Tile<BN>::STAGES][Tile<BN>::B_SLICE_BYTES];
  uint64_t full[Tile<BN>::STAGES], empty[Tile<BN>::STAGES];
  uint64_t acc_full, drain;
  uint32_t tmem_base;
  volatile int abort;
};
template <int BN>
constexpr size_t smem_bytes() { return sizeof(Smem<BN>) + 1024; }
static_assert(smem_bytes<16>() <= 227 * 1024 && smem_bytes<128>() <= 227 * 1024, "shared memory");

__device__ __forceinline__ bool wait_or_abort(volatile int& abort, uint64_t* bar, uint32_t parity) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(addr, parity)) return true;
    if (abort) return false;
    if (clock64() - t0 > kWaitBudgetCycles) {
      atomicOr(&g_tt_status, TT_ERR_TIMEOUT);
      abort = 1;
      return false;
    }
  }
}

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// (e, o) -> (e*c - o*s, e*s + o*c) with bf16 rounding after every operation (rope_append's
// rotate_pair).
__device__ __forceinline__ uint32_t rotate_pair(uint32_t pair, float c, float s) {
  const float e = bf16_lo(pair);
  const float o = bf16_hi(pair);
  const float r0 = bf16_round(e * c) - bf16_round(o * s);
  const float r1 = bf16_round(e * s) + bf16_round(o * c);
  return pack_bf16x2(r0, r1);
}

template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
qkv_rope_append_kernel(const __grid_constant__ CUtensorMap tm_h,
                       const __grid_constant__ CUtensorMap tm_w, const Params p) {
  using TL = Tile<BN>;
  constexpr int STAGES = TL::STAGES, SEG = TL::SEG;
  extern __shared__ uint8_t smem_raw[];
  Smem<BN>& s = *reinterpret_cast<Smem<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = static_cast<int>(blockIdx.x) * BN;  // output feature tile
  const int m0 = static_cast<int>(blockIdx.y) * BM;  // token row tile
  const int n_k = p.K / BK;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.acc_full, 1);
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, TL::TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == PRODUCER_WARP && lane == 0) {
    tma_prefetch_desc(&tm_h);
    tma_prefetch_desc(&tm_w);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == PRODUCER_WARP) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < n_k; ++kb) {
        const int st = kb % STAGES;
        if (kb >= STAGES && !wait_or_abort(s.abort, &s.empty[st], ((kb / STAGES) - 1) & 1)) break;
        mbar_arrive_expect_tx(&s.full[st], p.stage_tx_bytes);
        tma_load_2d(s.a[st], &tm_h, &s.full[st], kb * BK, m0);
        tma_load_2d(s.b[st], &tm_w, &s.full[st], kb * BK, n0);
        issued = kb + 1;
      }
      if (s.abort) {
        // Never leave while a TMA write into this CTA's shared memory is pending.
        for (int kb = max(0, issued - STAGES); kb < issued; ++kb)
          mbar_wait(&s.full[kb % STAGES], (kb / STAGES) & 1);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16(BM, BN, false);
      for (int kb = 0; kb < n_k; ++kb) {
        const int st = kb % STAGES;
        if (!wait_or_abort(s.abort, &s.full[st], (kb / STAGES) & 1)) break;
        tc_fence_after();
        const uint32_t a_addr = smem_u32(s.a[st]), b_addr = smem_u32(s.b[st]);
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          umma_ss(tmem, make_sdesc_sw128(a_addr + kk * 32, 16, 1024),
                  make_sdesc_sw128(b_addr + kk * 32, 16, 1024), idesc,
                  (kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&s.empty[st]);
      }
      umma_commit(&s.acc_full);
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0);
    }
  } else {
    // Epilogue: thread = token row m0 + r (TMEM lane r). Every SEG-column segment of the tile
    // lies inside one head of one part (q, k or v), at column `within` of that head.
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const bool ok = __all_sync(0xffffffffu, wait_or_abort(s.abort, &s.acc_full, 0));
    if (ok) {
      tc_fence_after();
      uint32_t acc[BN / SEG][SEG];
#pragma unroll
      for (int c = 0; c < BN / SEG; ++c) {
        if constexpr (SEG == 32) tmem_ld32(tmem + lane_base + c * 32, acc[c]);
        else tmem_ld16(tmem + lane_base + c * 16, acc[c]);
      }
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < BN / SEG; ++c) {
        if constexpr (SEG == 32) reg_fence(acc[c]);
        else reg_fence16(acc[c]);
      }
      const int m = m0 + r;
      const int part_cols = p.H * HD;
      const int part = n0 / part_cols;  // 0: q, 1: k, 2: v (BN divides 64 or 2 * 64 | part_cols)
      if (m < p.M) {
        const int b = m / p.T;
        const int t = m - b * p.T;
        const long long pos = (p.position_dev != nullptr ? *p.position_dev : p.position) + t;
        if (pos < 0 || pos >= p.capacity || pos >= p.table_len) {
          atomicOr(&g_tt_status, TT_ERR_RANGE);
        } else {
#pragma unroll
          for (int c = 0; c < BN / SEG; ++c) {
            const int col = n0 - part * part_cols + c * SEG;  // feature within the part
            const int head = col / HD, within = col % HD;
            uint32_t row[SEG / 2];
#pragma unroll
            for (int i = 0; i < SEG / 2; ++i)
              row[i] = pack_bf16x2(__uint_as_float(acc[c][2 * i]),
                                   __uint_as_float(acc[c][2 * i + 1]));
            if (part < 2) {
              const float4* c4 = reinterpret_cast<const float4*>(p.cos + pos * (HD / 2) + within / 2);
              const float4* s4 = reinterpret_cast<const float4*>(p.sin + pos * (HD / 2) + within / 2);
#pragma unroll
              for (int g = 0; g < SEG / 8; ++g) {
                const float4 cv = __ldg(c4 + g), sv = __ldg(s4 + g);
                row[4 * g] = rotate_pair(row[4 * g], bf16_round(cv.x), bf16_round(sv.x));
                row[4 * g + 1] = rotate_pair(row[4 * g + 1], bf16_round(cv.y), bf16_round(sv.y));
                row[4 * g + 2] = rotate_pair(row[4 * g + 2], bf16_round(cv.z), bf16_round(sv.z));
                row[4 * g + 3] = rotate_pair(row[4 * g + 3], bf16_round(cv.w), bf16_round(sv.w));
              }
            }
            __nv_bfloat16* dst;
            if (part == 0)
              dst = p.q_out + ((static_cast<long long>(b) * p.H + head) * p.T + t) * HD;
            else if (part == 1)
              dst = p.cache_k + b * p.ck_s0 + head * p.ck_s1 + pos * p.ck_s2;
            else
              dst = p.cache_v + b * p.cv_s0 + head * p.cv_s1 + pos * p.cv_s2;
            uint4* d4 = reinterpret_cast<uint4*>(dst + within);
#pragma unroll
            for (int i = 0; i < SEG / 8; ++i)
              d4[i] = make_uint4(row[4 * i], row[4 * i + 1], row[4 * i + 2], row[4 * i + 3]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TL::TMEM_COLS);
  }
}

}  // namespace qkv_rope
}  // namespace tt
