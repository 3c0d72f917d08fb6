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
// Both kernels stream 64-wide K slices of h and W with TMA (128-byte swizzle, no multicast)
// into a shared-memory ring, one thread issues tcgen05.mma (M = 128 token rows, N = BN
// features, both operands K-major) into TMEM, and four epilogue warps (thread = token row =
// TMEM lane) round, rotate and store each head's row segments. A feature tile of BN <= 128
// columns lies inside one of q, k, v (128 only with an even head count).
//
// * qkv_rope_splitk_kernel (one row tile, M <= 128: a decode step or a short prompt). A tcgen05
//   instruction costs a fixed ~56 cycles at N <= 64, so a CTA that walks the whole K range
//   spends K / 16 of them in series. Here a cluster of S CTAs shares one feature tile, each
//   taking a near-equal part of the K slices; every rank stores its FP32 partial sums into rank
//   0's shared memory (distributed shared memory, rows padded by 16 bytes so a warp's 16-byte
//   stores spread over the banks), one cluster barrier, and rank 0's four epilogue warps add
//   them in rank order (deterministic) and run the epilogue, one (row, 16-feature segment)
//   item per thread. The host picks S so that all clusters are resident at once. The h box
//   covers only the rows that exist (rounded up to 8); the MMA still reads 128 rows of A, and
//   accumulator rows beyond the box, computed from stale shared memory, are never stored.
// * qkv_rope_persistent_kernel (M > 128: prefill). One CTA per SM walks the (row tile, feature
//   tile) grid with a stride of the grid size; the K-slice ring runs on across tiles and the
//   accumulator alternates between two TMEM buffers, so the epilogue of one tile overlaps the
//   products of the next. Each epilogue thread loads its row's 32 cos / sin values before it
//   waits for the accumulator (one rotation table serves every head of the row), so the
//   epilogue is not a chain of L2 round trips.
//
// Rows past M are not stored. A device-held start position outside the cache or the table
// skips the row and sets TT_ERR_RANGE, as rope_append does. Every wait is bounded.
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
constexpr int MAX_SPLITS = 8;                    // portable cluster size

struct Params {
  int M, T, H, K;                 // M = B * T rows, H heads, K input features
  int n_tiles;                    // feature tiles (3 * H * 64 / BN)
  int m_tiles;                    // row tiles (persistent kernel)
  uint32_t stage_tx_bytes;        // bytes one stage's two TMA boxes deliver
  int red_rows;                   // split-K: rows of each partial-sum buffer (rows padded to 8)
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

template <int BN, int STAGES, int ACC>
struct alignas(1024) Smem {
  uint8_t a[STAGES][A_SLICE_BYTES];
  uint8_t b[STAGES][BN * BK * 2];
  uint64_t full[STAGES], empty[STAGES];
  uint64_t acc_full[ACC], acc_empty[ACC];
  uint64_t drain;
  uint32_t tmem_base;
  volatile int abort;
};

// Split-K: ring of 3 stages; the partial sums follow the fixed part.
constexpr int SK_STAGES = 3;
template <int BN>
using SmemSK = Smem<BN, SK_STAGES, 1>;
// Persistent: about 192 KiB of stages, two accumulators.
template <int BN>
struct Pers {
  static constexpr int STAGES = BN == 128 ? 6 : 8;
};
template <int BN>
using SmemP = Smem<BN, Pers<BN>::STAGES, 2>;

template <int BN>
constexpr size_t splitk_fixed_bytes() { return sizeof(SmemSK<BN>) + 1024; }
template <int BN>
constexpr size_t persistent_smem_bytes() { return sizeof(SmemP<BN>) + 1024; }
static_assert(persistent_smem_bytes<128>() <= 227 * 1024 &&
              persistent_smem_bytes<64>() <= 227 * 1024, "shared memory");

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

// Packed bf16 arithmetic (round to nearest even, one rounding per operation).
__device__ __forceinline__ uint32_t bmul2(uint32_t a, uint32_t b) {
  uint32_t d;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}
__device__ __forceinline__ uint32_t bfma2(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t d;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
constexpr uint32_t kMinusPlusOne = 0x3F80BF80u;  // bf16x2 (lo -1.0, hi +1.0)

// (e, o) -> (e*c - o*s, o*c + e*s) on a bf16x2 pair, with the bf16 steps of rope_append (each
// product rounded to bf16, then the difference / sum rounded): (e*c, o*c) and (o*s, e*s) by two
// packed multiplies, then one packed FMA with (-1, +1) forms both results with one rounding
// each. cc = (c, c) and ss = (s, s) hold the bf16-rounded cos / sin.
__device__ __forceinline__ uint32_t rotate_pair2(uint32_t eo, uint32_t cc, uint32_t ss) {
  const uint32_t oe = __byte_perm(eo, 0, 0x1032);
  return bfma2(bmul2(oe, ss), kMinusPlusOne, bmul2(eo, cc));
}

// Where token row m goes: its batch / step and cache position; ok is false for rows past M and
// (flagging TT_ERR_RANGE) for positions outside the cache or the table.
struct RowDest {
  int b, t;
  long long pos;
  bool ok;
};

__device__ __forceinline__ RowDest row_dest(const Params& p, int m) {
  RowDest d{0, 0, 0, false};
  if (m >= p.M) return d;
  d.b = m / p.T;
  d.t = m - d.b * p.T;
  d.pos = (p.position_dev != nullptr ? *p.position_dev : p.position) + d.t;
  if (d.pos < 0 || d.pos >= p.capacity || d.pos >= p.table_len) {
    atomicOr(&g_tt_status, TT_ERR_RANGE);
    return d;
  }
  d.ok = true;
  return d;
}

// cos / sin of rotation pairs [i0, i0 + N) of position pos (N % 4 == 0), rounded to bf16 and
// duplicated into both halves of a bf16x2 word.
template <int N>
__device__ __forceinline__ void load_rotation(const Params& p, long long pos, int i0,
                                              uint32_t (&cc)[N], uint32_t (&ss)[N]) {
  const float4* c4 = reinterpret_cast<const float4*>(p.cos + pos * (HD / 2) + i0);
  const float4* s4 = reinterpret_cast<const float4*>(p.sin + pos * (HD / 2) + i0);
#pragma unroll
  for (int g = 0; g < N / 4; ++g) {
    const float4 cv = __ldg(c4 + g), sv = __ldg(s4 + g);
    cc[4 * g] = pack_bf16x2(cv.x, cv.x); cc[4 * g + 1] = pack_bf16x2(cv.y, cv.y);
    cc[4 * g + 2] = pack_bf16x2(cv.z, cv.z); cc[4 * g + 3] = pack_bf16x2(cv.w, cv.w);
    ss[4 * g] = pack_bf16x2(sv.x, sv.x); ss[4 * g + 1] = pack_bf16x2(sv.y, sv.y);
    ss[4 * g + 2] = pack_bf16x2(sv.z, sv.z); ss[4 * g + 3] = pack_bf16x2(sv.w, sv.w);
  }
}

// Store SEG features [col, col + SEG) (col within the part, SEG | 64) of one token row: round to
// bf16, and for q and k rotate with the preloaded pairs cc / ss (pair i of the segment).
template <int SEG>
__device__ __forceinline__ void store_rotated(const Params& p, const RowDest& d, int part, int col,
                                              const float (&v)[SEG], const uint32_t* cc,
                                              const uint32_t* ss) {
  const int head = col / HD, within = col % HD;
  uint32_t row[SEG / 2];
#pragma unroll
  for (int i = 0; i < SEG / 2; ++i) {
    row[i] = pack_bf16x2(v[2 * i], v[2 * i + 1]);
    if (part < 2) row[i] = rotate_pair2(row[i], cc[i], ss[i]);
  }
  __nv_bfloat16* dst;
  if (part == 0)
    dst = p.q_out + ((static_cast<long long>(d.b) * p.H + head) * p.T + d.t) * HD;
  else if (part == 1)
    dst = p.cache_k + d.b * p.ck_s0 + head * p.ck_s1 + d.pos * p.ck_s2;
  else
    dst = p.cache_v + d.b * p.cv_s0 + head * p.cv_s1 + d.pos * p.cv_s2;
  uint4* d4 = reinterpret_cast<uint4*>(dst + within);
#pragma unroll
  for (int i = 0; i < SEG / 8; ++i)
    d4[i] = make_uint4(row[4 * i], row[4 * i + 1], row[4 * i + 2], row[4 * i + 3]);
}

template <int SEG>
__device__ __forceinline__ void tmem_load_seg(uint32_t taddr, uint32_t (&r)[SEG]) {
  if constexpr (SEG == 32) tmem_ld32(taddr, r);
  else tmem_ld16(taddr, r);
}
template <int SEG>
__device__ __forceinline__ void fence_seg(uint32_t (&r)[SEG]) {
  if constexpr (SEG == 32) reg_fence(r);
  else reg_fence16(r);
}

__device__ __forceinline__ void issue_k_slice(uint32_t tmem_acc, uint32_t a_addr, uint32_t b_addr,
                                              uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < BK / 16; ++kk)
    umma_ss(tmem_acc, make_sdesc_sw128(a_addr + kk * 32, 16, 1024),
            make_sdesc_sw128(b_addr + kk * 32, 16, 1024), idesc, (accumulate || kk > 0) ? 1u : 0u);
}

// ------------------------------------------------------------------------------ split-K
// Grid (S, n_tiles), cluster (S, 1, 1): CTA rank z of the cluster takes K slices
// [z * n_k / S, (z + 1) * n_k / S) of feature tile blockIdx.y. Dynamic shared memory: the fixed
// part, then S partial-sum buffers [red_rows][BN + 4] FP32 (used in rank 0 only).
template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
qkv_rope_splitk_kernel(const __grid_constant__ CUtensorMap tm_h,
                       const __grid_constant__ CUtensorMap tm_w, const Params p) {
  constexpr int SEG = BN < 32 ? BN : 32;
  constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  constexpr int RED_STRIDE = BN + 4;  // floats per partial-sum row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~uintptr_t(1023));
  SmemSK<BN>& s = *reinterpret_cast<SmemSK<BN>*>(base);
  float* red = reinterpret_cast<float*>(base + sizeof(SmemSK<BN>));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int splits = static_cast<int>(gridDim.x);
  const int rank = static_cast<int>(blockIdx.x);  // == %cluster_ctarank for cluster (S, 1, 1)
  const int n0 = static_cast<int>(blockIdx.y) * BN;
  const int n_k = p.K / BK;
  const int kb0 = rank * n_k / splits, kb1 = (rank + 1) * n_k / splits;

  if (threadIdx.x == 0) {
    for (int i = 0; i < SK_STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    mbar_init(&s.acc_full[0], 1);
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
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
  const int quarter = warp & 3;
  const int r = quarter * 32 + lane;
  const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
  bool acc_ok = false;

  if (warp == PRODUCER_WARP) {
    if (lane == 0) {
      int issued = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0, st = i % SK_STAGES;
        if (i >= SK_STAGES && !wait_or_abort(s.abort, &s.empty[st], ((i / SK_STAGES) - 1) & 1))
          break;
        mbar_arrive_expect_tx(&s.full[st], p.stage_tx_bytes);
        tma_load_2d(s.a[st], &tm_h, &s.full[st], kb * BK, 0);
        tma_load_2d(s.b[st], &tm_w, &s.full[st], kb * BK, n0);
        issued = i + 1;
      }
      if (s.abort) {
        // Never leave while a TMA write into this CTA's shared memory is pending.
        for (int i = max(0, issued - SK_STAGES); i < issued; ++i)
          mbar_wait(&s.full[i % SK_STAGES], (i / SK_STAGES) & 1);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16(BM, BN, false);
      for (int kb = kb0; kb < kb1; ++kb) {
        const int i = kb - kb0, st = i % SK_STAGES;
        if (!wait_or_abort(s.abort, &s.full[st], (i / SK_STAGES) & 1)) break;
        tc_fence_after();
        issue_k_slice(tmem, smem_u32(s.a[st]), smem_u32(s.b[st]), idesc, i > 0);
        umma_commit(&s.empty[st]);
      }
      umma_commit(&s.acc_full[0]);
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0);
    }
  }

  // Rank 0's epilogue threads: first (row, 16-feature segment) item of this thread, its row's
  // destination and rotation pairs, fetched while the products run.
  const int part_cols = p.H * HD;
  const int part = n0 / part_cols;
  const int items = p.red_rows * (BN / 16);
  const int et = static_cast<int>(threadIdx.x) - EPI_WARP0 * 32;  // epilogue thread 0..127
  uint32_t c0[8] = {}, s0[8] = {};
  RowDest d0{0, 0, 0, false};
  if (rank == 0 && warp >= EPI_WARP0 && et < items) {
    d0 = row_dest(p, et % p.red_rows);
    if (d0.ok && part < 2)
      load_rotation<8>(p, d0.pos, ((n0 - part * part_cols) % HD + (et / p.red_rows) * 16) / 2, c0,
                       s0);
  }

  if (warp >= EPI_WARP0) {
    acc_ok = __all_sync(0xffffffffu, wait_or_abort(s.abort, &s.acc_full[0], 0));
    if (acc_ok) {
      // This rank's partial sums to rank 0, rows [row][BN + 4] (lane = row).
      const uint32_t dst0 = map_to_rank(smem_u32(red), 0) +
                            static_cast<uint32_t>((rank * p.red_rows + r) * RED_STRIDE) * 4u;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < BN / SEG; ++c) {
        uint32_t v[SEG];
        tmem_load_seg<SEG>(tmem + lane_base + c * SEG, v);
        tmem_wait_ld();
        fence_seg<SEG>(v);
        if (r < p.red_rows) {
#pragma unroll
          for (int i = 0; i < SEG; i += 4)
            st_cluster_v4(dst0 + static_cast<uint32_t>(c * SEG + i) * 4u, v[i], v[i + 1],
                          v[i + 2], v[i + 3]);
        }
      }
    }
  }

  // Every thread of every CTA: all partial sums are in rank 0's shared memory after this.
  __syncwarp();
  cluster_sync();

  if (warp >= EPI_WARP0 && rank == 0 && acc_ok) {
    for (int it = et; it < items; it += 4 * 32) {
      const int row = it % p.red_rows, seg = it / p.red_rows;
      RowDest d = d0;
      uint32_t c[8], sn[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) { c[i] = c0[i]; sn[i] = s0[i]; }
      const int col = n0 - part * part_cols + seg * 16;
      if (it != et) {
        d = row_dest(p, row);
        if (d.ok && part < 2) load_rotation<8>(p, d.pos, (col % HD) / 2, c, sn);
      }
      if (!d.ok) continue;
      float f[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) f[i] = 0.f;
      for (int z = 0; z < splits; ++z) {
        const float4* src = reinterpret_cast<const float4*>(
            red + static_cast<size_t>(z * p.red_rows + row) * RED_STRIDE + seg * 16);
#pragma unroll
        for (int g = 0; g < 4; ++g) {
          const float4 q = src[g];
          f[4 * g] += q.x; f[4 * g + 1] += q.y; f[4 * g + 2] += q.z; f[4 * g + 3] += q.w;
        }
      }
      store_rotated<16>(p, d, part, col, f, c, sn);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// --------------------------------------------------------------------------- persistent
// Grid: min(tiles, SMs) CTAs; CTA c takes tiles c, c + grid, ... (feature tile fastest).
template <int BN>
__global__ void __launch_bounds__(THREADS, 1)
qkv_rope_persistent_kernel(const __grid_constant__ CUtensorMap tm_h,
                           const __grid_constant__ CUtensorMap tm_w, const Params p) {
  constexpr int STAGES = Pers<BN>::STAGES;
  constexpr int SEG = 32;
  constexpr uint32_t TMEM_COLS = 2 * BN;
  extern __shared__ uint8_t smem_raw[];
  SmemP<BN>& s = *reinterpret_cast<SmemP<BN>*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_k = p.K / BK;
  const int tiles = p.m_tiles * p.n_tiles;
  const int first = static_cast<int>(blockIdx.x), stride = static_cast<int>(gridDim.x);

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&s.acc_full[a], 1);
      mbar_init(&s.acc_empty[a], 4);  // the four epilogue warps
    }
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
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
      int g = 0;  // slices issued by this CTA (ring position)
      bool ok = true;
      for (int tile = first; ok && tile < tiles; tile += stride) {
        const int m0 = (tile / p.n_tiles) * BM, n0 = (tile % p.n_tiles) * BN;
        for (int kb = 0; kb < n_k; ++kb, ++g) {
          const int st = g % STAGES;
          if (g >= STAGES && !wait_or_abort(s.abort, &s.empty[st], ((g / STAGES) - 1) & 1)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&s.full[st], p.stage_tx_bytes);
          tma_load_2d(s.a[st], &tm_h, &s.full[st], kb * BK, m0);
          tma_load_2d(s.b[st], &tm_w, &s.full[st], kb * BK, n0);
        }
      }
      if (s.abort) {
        for (int i = max(0, g - STAGES); i < g; ++i) mbar_wait(&s.full[i % STAGES], (i / STAGES) & 1);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc = make_idesc_bf16(BM, BN, false);
      int g = 0, local = 0;
      bool ok = true;
      for (int tile = first; ok && tile < tiles; tile += stride, ++local) {
        const int a = local & 1;
        // The epilogue has read this accumulator's previous tile.
        if (local >= 2 && !wait_or_abort(s.abort, &s.acc_empty[a], ((local >> 1) - 1) & 1)) break;
        tc_fence_after();
        const uint32_t acc = tmem + a * BN;
        for (int kb = 0; kb < n_k; ++kb, ++g) {
          const int st = g % STAGES;
          if (!wait_or_abort(s.abort, &s.full[st], (g / STAGES) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_k_slice(acc, smem_u32(s.a[st]), smem_u32(s.b[st]), idesc, kb > 0);
          umma_commit(&s.empty[st]);
        }
        if (ok) umma_commit(&s.acc_full[a]);
      }
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0);
    }
  } else {
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int part_cols = p.H * HD;
    int local = 0;
    for (int tile = first; tile < tiles; tile += stride, ++local) {
      const int a = local & 1;
      const int m0 = (tile / p.n_tiles) * BM, n0 = (tile % p.n_tiles) * BN;
      const int part = n0 / part_cols;
      // The row's destination and its 32 rotation pairs (the same for every head), fetched
      // before the accumulator is ready.
      const RowDest d = row_dest(p, m0 + r);
      uint32_t c[HD / 2], sn[HD / 2];
      if (d.ok && part < 2) load_rotation<HD / 2>(p, d.pos, 0, c, sn);
      if (!__all_sync(0xffffffffu, wait_or_abort(s.abort, &s.acc_full[a], (local >> 1) & 1)))
        break;
      tc_fence_after();
      // One head (64 columns) at a time: two 32-column loads, then round / rotate / store.
#pragma unroll 1
      for (int hc = 0; hc < BN / HD; ++hc) {
        uint32_t v0[SEG], v1[SEG];
        tmem_ld32(tmem + lane_base + a * BN + hc * HD, v0);
        tmem_ld32(tmem + lane_base + a * BN + hc * HD + SEG, v1);
        tmem_wait_ld();
        reg_fence(v0);
        reg_fence(v1);
        if (hc == BN / HD - 1) {
          // Accumulator fully read: the MMA warp may start the tile after next in it.
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.acc_empty[a]);
        }
        if (d.ok) {
          float f[HD];
#pragma unroll
          for (int i = 0; i < SEG; ++i) {
            f[i] = __uint_as_float(v0[i]);
            f[SEG + i] = __uint_as_float(v1[i]);
          }
          store_rotated<HD>(p, d, part, n0 - part * part_cols + hc * HD, f, c, sn);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace qkv_rope
}  // namespace tt
