// Deterministic BF16 causal attention backward for sm_100a: the same results contract as the
// fused kernel in backward_sm100.cuh (reference semantics: Tiny-transformer
// csrc/attention/attention.cu:161-234), with every sum accumulated in a fixed order, so that
// repeated calls give bit-identical dQ, dK and dV. It is the path taken under
// torch.use_deterministic_algorithms(True), like the reference's own backward (which uses no
// atomics); the fused kernel adds dQ contributions from different CTAs with reduce-adds in
// timing-dependent order.
//   D_i   = sum_d dO[i, d] * O[i, d]                           (FP32)
//   P_ij  = exp(scale * q_i.k_j - LSE_i) on visible pairs, else 0 (FP32)
//   dS_ij = P_ij * (dO_i.v_j - D_i)                            (FP32)
//   dV_j  = sum_i bf16(P_ij) dO_i,   dK_j = scale * sum_i bf16(dS_ij) q_i,
//   dQ_i  = scale * sum_j bf16(dS_ij) k_j                      (FP32 accumulate, BF16 out)
// with key j visible to query i iff j <= i + past_len (Tk == Tq + past_len), scale = 1/8.
//
// Three kernels, in stream order:
// * bwd_preprocess_kernel: D, eight lanes per query row (16-byte loads of dO and O).
// * bwd_dq_kernel: one CTA per (b, h, 128-row query tile), stepping over 64-key tiles.
//   tcgen05: S = Q.K^T and dP = dO.V^T (SS, M = 128, N = 64, into TMEM); the elementwise warps
//   (thread = query row = TMEM lane) read them and write bf16 dS over the S columns they have
//   just read; then dQ += dS.K (TS, A from TMEM). TMEM: S/dS [0,64), dP [64,128), dQ [128,192).
// * bwd_dkdv_kernel: one CTA per (b, h, 128-key tile), stepping over 64-row query tiles, in
//   transposed form so that keys are the TMEM lanes: S^T = K.Q^T, dP^T = V.dO^T; the
//   elementwise warps (thread = key row) write bf16 P^T over S^T and dS^T over dP^T, then
//   dV += P^T.dO and dK += dS^T.Q (TS). Per-query LSE and D come from shared memory (broadcast
//   reads). TMEM: S^T/P^T [0,64), dP^T/dS^T [64,128), dV [128,192), dK [192,256).
// Each step of a CTA is a serial chain (scores -> elementwise -> accumulation). With 256 TMEM
// columns and ~80 KB of shared memory per CTA, two CTAs share an SM and overlap their chains.
// Roles: warps 0-3 elementwise + epilogue, warp 4 TMA producer (all lanes stage LSE/D in the
// dK/dV kernel), warp 5 tcgen05 issuer (one thread). Every mbarrier wait is bounded
// (TT_ERR_TIMEOUT + abort flag), as in the forward kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace tt {
namespace backward_det {

constexpr int TILE = 128;  // rows of the CTA's own tile (UMMA M): query rows or keys
constexpr int STEP = 64;   // rows of the tile stepped over (UMMA N of the scores)
constexpr int HD = 64;
constexpr int STAGES = 3;
constexpr int THREADS = 192;  // 4 elementwise warps, TMA warp, issuer warp
constexpr int LOAD_WARP = 4, MMA_WARP = 5;
constexpr uint32_t TILE_BYTES = TILE * HD * 2;  // 16 KiB
constexpr uint32_t STEP_BYTES = STEP * HD * 2;  // 8 KiB
constexpr uint32_t TMEM_COLS = 256;
constexpr float SCALE = 0.125f;
constexpr float LOG2E = 1.4426950408889634f;

struct Params {
  int B, H, Tq, Tk, past_len;
  int n_tiles;              // query tiles (dQ kernel) or key tiles (dK/dV kernel) of TILE rows
  const float* lse;         // contiguous [B, H, Tq], natural log
  const float* D;           // contiguous [B, H, Tq]
  __nv_bfloat16* out0;      // dQ (dQ kernel) or dK (dK/dV kernel), contiguous
  __nv_bfloat16* out1;      // dV (dK/dV kernel), contiguous
};

// ------------------------------------------------------------------ preprocess
struct PreParams {
  long long rows;            // B * H * Tq
  const __nv_bfloat16* dO;   // contiguous [rows, 64]
  const __nv_bfloat16* O;
  float* D;
};

// Eight lanes per row, 16-byte loads: a warp covers four rows, a block of 256 threads 32.
constexpr int PRE_ROWS_PER_BLOCK = 32;

__global__ void __launch_bounds__(256) bwd_preprocess_kernel(const PreParams p) {
  const long long row =
      static_cast<long long>(blockIdx.x) * PRE_ROWS_PER_BLOCK + (threadIdx.x >> 3);
  const int part = threadIdx.x & 7;  // 8 features per lane
  float sum = 0.f;
  if (row < p.rows) {
    const uint4 a = reinterpret_cast<const uint4*>(p.dO + row * HD)[part];
    const uint4 o = reinterpret_cast<const uint4*>(p.O + row * HD)[part];
    sum = bf16_lo(a.x) * bf16_lo(o.x) + bf16_hi(a.x) * bf16_hi(o.x) +
          bf16_lo(a.y) * bf16_lo(o.y) + bf16_hi(a.y) * bf16_hi(o.y) +
          bf16_lo(a.z) * bf16_lo(o.z) + bf16_hi(a.z) * bf16_hi(o.z) +
          bf16_lo(a.w) * bf16_lo(o.w) + bf16_hi(a.w) * bf16_hi(o.w);
  }
  // Reduce over the eight lanes of the row (all 32 lanes take part in every shuffle).
#pragma unroll
  for (int off = 4; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (part == 0 && row < p.rows) p.D[row] = sum;
}

// ------------------------------------------------------------------ shared pieces
struct alignas(1024) SmemQ {  // dQ kernel
  uint8_t q[TILE_BYTES];
  uint8_t dO[TILE_BYTES];
  uint8_t k[STAGES][STEP_BYTES];
  uint8_t v[STAGES][STEP_BYTES];
  uint64_t qd_full;
  uint64_t kv_full[STAGES], kv_empty[STAGES];
  uint64_t s_full, s_free, ds_ready, dq_done, drain;
  uint32_t tmem_base;
  volatile int abort;
};

struct alignas(1024) SmemKV {  // dK/dV kernel
  uint8_t k[TILE_BYTES];
  uint8_t v[TILE_BYTES];
  uint8_t q[STAGES][STEP_BYTES];
  uint8_t dO[STAGES][STEP_BYTES];
  float lse2[STAGES][STEP];  // LSE * log2(e) per query row of the stage (+inf past Tq)
  float d[STAGES][STEP];
  uint64_t kv_full;
  uint64_t q_full[STAGES], q_empty[STAGES];
  uint64_t st_full, st_free, pd_ready, acc_done, drain;
  uint32_t tmem_base;
  volatile int abort;
};

constexpr size_t kSmemQ = sizeof(SmemQ) + 1024;
constexpr size_t kSmemKV = sizeof(SmemKV) + 1024;
static_assert(2 * kSmemQ <= 228 * 1024 && 2 * kSmemKV <= 228 * 1024,
              "two CTAs per SM must fit in shared memory");

template <class S>
__device__ __forceinline__ bool wait_or_abort(S& s, uint64_t* bar, uint32_t parity) {
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

template <class S>
__device__ __forceinline__ bool warp_wait(S& s, uint64_t* bar, uint32_t parity) {
  const bool ok = wait_or_abort(s, bar, parity);
  return __all_sync(0xffffffffu, ok);
}

// D = A.B^T with A, B both K-major 128-byte-swizzled tiles of 64 features (4 k-steps of 16).
__device__ __forceinline__ void issue_scores(uint32_t tmem_d, uint32_t a_addr, uint32_t b_addr,
                                             uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk)
    umma_ss(tmem_d, make_sdesc_sw128(a_addr + kk * 32, 16, 1024),
            make_sdesc_sw128(b_addr + kk * 32, 16, 1024), idesc, kk > 0 ? 1u : 0u);
}

// D += A.B with A = bf16 pairs in TMEM over STEP rows of K, laid out by the elementwise warps
// as chunk c (K rows [32c, 32c + 32)) at TMEM columns [32c, 32c + 16) of its region; B = a
// STEP x 64 tile, MN-major (16 K rows x 128 B = 2048 B per k-step).
__device__ __forceinline__ void issue_accumulate(uint32_t tmem_d, uint32_t tmem_a, uint32_t b_addr,
                                                 uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < STEP / 16; ++kk)
    umma_ts(tmem_d, tmem_a + 32 * (kk >> 1) + 8 * (kk & 1),
            make_sdesc_sw128(b_addr + kk * 2048, 8192, 1024), idesc,
            (accumulate || kk > 0) ? 1u : 0u);
}

__device__ __forceinline__ void store_row_bf16(__nv_bfloat16* dst, const uint32_t (&acc)[32],
                                               float scale) {
  uint32_t packed[16];
#pragma unroll
  for (int e = 0; e < 16; ++e)
    packed[e] = pack_bf16x2(__uint_as_float(acc[2 * e]) * scale,
                            __uint_as_float(acc[2 * e + 1]) * scale);
  uint4* d4 = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int e = 0; e < 4; ++e)
    d4[e] = make_uint4(packed[4 * e], packed[4 * e + 1], packed[4 * e + 2], packed[4 * e + 3]);
}

// ------------------------------------------------------------------ dQ kernel
__global__ void __launch_bounds__(THREADS, 2)
bwd_dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
              const Params p) {
  extern __shared__ uint8_t smem_raw[];
  SmemQ& s = *reinterpret_cast<SmemQ*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                       ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int qt = p.n_tiles - 1 - static_cast<int>(blockIdx.x / BH);  // heaviest tiles first
  const int bh = static_cast<int>(blockIdx.x % BH);
  const int b = bh / p.H, h = bh % p.H;
  const int q0 = qt * TILE;
  const long long kend =
      min(static_cast<long long>(p.Tk), static_cast<long long>(q0) + TILE + p.past_len);
  const int n_kv = static_cast<int>((kend + STEP - 1) / STEP);  // key steps this tile sees
  constexpr uint32_t T_S = 0, T_DP = 64, T_DQ = 128;

  if (threadIdx.x == 0) {
    mbar_init(&s.qd_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], 1);
    }
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_free, 4);
    mbar_init(&s.ds_ready, 4);
    mbar_init(&s.dq_done, 1);
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == LOAD_WARP) {
    if (lane == 0) {
      int issued = 0;
      mbar_arrive_expect_tx(&s.qd_full, 2 * TILE_BYTES);
      tma_load_4d(s.q, &tm_q, &s.qd_full, 0, q0, h, b);
      tma_load_4d(s.dO, &tm_do, &s.qd_full, 0, q0, h, b);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % STAGES;
        if (j >= STAGES && !wait_or_abort(s, &s.kv_empty[st], ((j / STAGES) - 1) & 1)) break;
        mbar_arrive_expect_tx(&s.kv_full[st], 2 * STEP_BYTES);
        tma_load_4d(s.k[st], &tm_k, &s.kv_full[st], 0, j * STEP, h, b);
        tma_load_4d(s.v[st], &tm_v, &s.kv_full[st], 0, j * STEP, h, b);
        issued = j + 1;
      }
      if (s.abort) {
        mbar_wait(&s.qd_full, 0);
        for (int j = max(0, issued - STAGES); j < issued; ++j)
          mbar_wait(&s.kv_full[j % STAGES], (j / STAGES) & 1);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(TILE, STEP, false);
      const uint32_t idesc_o = make_idesc_bf16(TILE, HD, true);
      const uint32_t q_addr = smem_u32(s.q), do_addr = smem_u32(s.dO);
      bool ok = wait_or_abort(s, &s.qd_full, 0);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % STAGES;
        if (!wait_or_abort(s, &s.kv_full[st], (j / STAGES) & 1)) break;
        if (j > 0 && !wait_or_abort(s, &s.s_free, (j - 1) & 1)) break;
        tc_fence_after();
        issue_scores(tmem + T_S, q_addr, smem_u32(s.k[st]), idesc_s);
        issue_scores(tmem + T_DP, do_addr, smem_u32(s.v[st]), idesc_s);
        umma_commit(&s.s_full);
        if (!wait_or_abort(s, &s.ds_ready, j & 1)) break;
        tc_fence_after();
        issue_accumulate(tmem + T_DQ, tmem + T_S, smem_u32(s.k[st]), idesc_o, j > 0);
        umma_commit(&s.dq_done);
        umma_commit(&s.kv_empty[st]);
      }
      // All MMAs issued by this thread have completed once `drain` flips.
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0);
    }
  } else {
    // Elementwise warps: thread = query row r of the tile = TMEM lane.
    const int wq = warp, r = wq * 32 + lane;
    const int row = q0 + r;
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const size_t ridx = static_cast<size_t>(bh) * p.Tq + static_cast<size_t>(row);
    const float lse2 = row < p.Tq ? p.lse[ridx] * LOG2E : INFINITY;
    const float drow = row < p.Tq ? p.D[ridx] : 0.f;
    const long long row_limit = static_cast<long long>(row) + p.past_len;
    const long long tile_limit = static_cast<long long>(q0) + p.past_len;
    const float sl2 = SCALE * LOG2E;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      if (!warp_wait(s, &s.s_full, j & 1)) { ok = false; break; }
      // dS overwrites S, which the previous dQ += dS.K may still be reading.
      if (j > 0 && !warp_wait(s, &s.dq_done, (j - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      const long long kv0 = static_cast<long long>(j) * STEP;
      const bool masked = kv0 + STEP - 1 > tile_limit;
#pragma unroll
      for (int c = 0; c < STEP / 32; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld32(tmem + lane_base + T_S + c * 32, sr);
        tmem_ld32(tmem + lane_base + T_DP + c * 32, dr);
        tmem_wait_ld();
        reg_fence(sr);
        reg_fence(dr);
        uint32_t ds[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float dv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = 2 * e + u;
            float pp = ex2_approx(__uint_as_float(sr[col]) * sl2 - lse2);
            if (masked && kv0 + c * 32 + col > row_limit) pp = 0.f;
            dv[u] = pp * (__uint_as_float(dr[col]) - drow);
          }
          ds[e] = pack_bf16x2(dv[0], dv[1]);
        }
        tmem_st16(tmem + lane_base + T_S + c * 32, ds);  // over S columns this thread has read
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.s_free);
        mbar_arrive(&s.ds_ready);
      }
    }
    if (ok && warp_wait(s, &s.dq_done, (n_kv - 1) & 1)) {
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t acc[32];
        tmem_ld32(tmem + lane_base + T_DQ + c * 32, acc);
        tmem_wait_ld();
        reg_fence(acc);
        if (row < p.Tq) store_row_bf16(p.out0 + ridx * HD + c * 32, acc, SCALE);
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

// ------------------------------------------------------------------ dK/dV kernel
__global__ void __launch_bounds__(THREADS, 2)
bwd_dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                const Params p) {
  extern __shared__ uint8_t smem_raw[];
  SmemKV& s = *reinterpret_cast<SmemKV*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                         ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int kt = static_cast<int>(blockIdx.x / BH);  // low key tiles see the most queries
  const int bh = static_cast<int>(blockIdx.x % BH);
  const int b = bh / p.H, h = bh % p.H;
  const int k0 = kt * TILE;
  // Query steps (of STEP rows) that see some key of this tile: from the step holding query
  // k0 - past_len on; the last query row sees every key, so there is at least one.
  const int qs0 = static_cast<int>(max(0LL, static_cast<long long>(k0) - p.past_len) / STEP);
  const int n_q = (p.Tq + STEP - 1) / STEP - qs0;
  constexpr uint32_t T_ST = 0, T_DPT = 64, T_DV = 128, T_DK = 192;

  if (threadIdx.x == 0) {
    mbar_init(&s.kv_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 1);
    }
    mbar_init(&s.st_full, 1);
    mbar_init(&s.st_free, 4);
    mbar_init(&s.pd_ready, 4);
    mbar_init(&s.acc_done, 1);
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == LOAD_WARP) {
    int issued = 0;
    if (lane == 0) {
      mbar_arrive_expect_tx(&s.kv_full, 2 * TILE_BYTES);
      tma_load_4d(s.k, &tm_k, &s.kv_full, 0, k0, h, b);
      tma_load_4d(s.v, &tm_v, &s.kv_full, 0, k0, h, b);
    }
    for (int i = 0; i < n_q; ++i) {
      const int st = i % STAGES;
      const int q0 = (qs0 + i) * STEP;
      if (i >= STAGES && !warp_wait(s, &s.q_empty[st], ((i / STAGES) - 1) & 1)) break;
      // Per-query LSE (log2 units) and D of this step; rows past Tq get +inf / 0, so their
      // probabilities are exactly zero.
#pragma unroll
      for (int e = 0; e < STEP / 32; ++e) {
        const int rr = e * 32 + lane;
        const int q = q0 + rr;
        const size_t idx = static_cast<size_t>(bh) * p.Tq + static_cast<size_t>(q);
        s.lse2[st][rr] = q < p.Tq ? p.lse[idx] * LOG2E : INFINITY;
        s.d[st][rr] = q < p.Tq ? p.D[idx] : 0.f;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&s.q_full[st], 2 * STEP_BYTES);
        tma_load_4d(s.q[st], &tm_q, &s.q_full[st], 0, q0, h, b);
        tma_load_4d(s.dO[st], &tm_do, &s.q_full[st], 0, q0, h, b);
      }
      issued = i + 1;
    }
    if (lane == 0 && s.abort) {
      mbar_wait(&s.kv_full, 0);
      for (int i = max(0, issued - STAGES); i < issued; ++i)
        mbar_wait(&s.q_full[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(TILE, STEP, false);
      const uint32_t idesc_o = make_idesc_bf16(TILE, HD, true);
      const uint32_t k_addr = smem_u32(s.k), v_addr = smem_u32(s.v);
      bool ok = wait_or_abort(s, &s.kv_full, 0);
      for (int i = 0; ok && i < n_q; ++i) {
        const int st = i % STAGES;
        if (!wait_or_abort(s, &s.q_full[st], (i / STAGES) & 1)) break;
        if (i > 0 && !wait_or_abort(s, &s.st_free, (i - 1) & 1)) break;
        tc_fence_after();
        issue_scores(tmem + T_ST, k_addr, smem_u32(s.q[st]), idesc_s);
        issue_scores(tmem + T_DPT, v_addr, smem_u32(s.dO[st]), idesc_s);
        umma_commit(&s.st_full);
        if (!wait_or_abort(s, &s.pd_ready, i & 1)) break;
        tc_fence_after();
        issue_accumulate(tmem + T_DV, tmem + T_ST, smem_u32(s.dO[st]), idesc_o, i > 0);
        issue_accumulate(tmem + T_DK, tmem + T_DPT, smem_u32(s.q[st]), idesc_o, i > 0);
        umma_commit(&s.acc_done);
        umma_commit(&s.q_empty[st]);
      }
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0);
    }
  } else {
    // Elementwise warps: thread = key row of the tile = TMEM lane.
    const int wq = warp, r = wq * 32 + lane;
    const int key = k0 + r;
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const float sl2 = SCALE * LOG2E;
    bool ok = true;
    for (int i = 0; i < n_q; ++i) {
      const int st = i % STAGES;
      const long long q0 = static_cast<long long>(qs0 + i) * STEP;
      if (!warp_wait(s, &s.st_full, i & 1)) { ok = false; break; }
      // P^T / dS^T overwrite S^T / dP^T, which the previous accumulation may still read.
      if (i > 0 && !warp_wait(s, &s.acc_done, (i - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      // Pair (key, q) is visible iff key <= q + past_len; only steps crossing the diagonal mask.
      const bool masked = static_cast<long long>(k0) + TILE - 1 > q0 + p.past_len;
#pragma unroll
      for (int c = 0; c < STEP / 32; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld32(tmem + lane_base + T_ST + c * 32, sr);
        tmem_ld32(tmem + lane_base + T_DPT + c * 32, dr);
        tmem_wait_ld();
        reg_fence(sr);
        reg_fence(dr);
        uint32_t pk[16], ds[16];
        // Per-query LSE and D through explicit shared loads (a re-aligned Smem& would make
        // them generic loads).
        const uint32_t lse_addr = smem_u32(&s.lse2[st][c * 32]);
        const uint32_t d_addr = smem_u32(&s.d[st][c * 32]);
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float4 l4 = lds_f4(lse_addr + 8 * e);
          const float4 d4 = lds_f4(d_addr + 8 * e);
          const float lv[4] = {l4.x, l4.y, l4.z, l4.w}, dl[4] = {d4.x, d4.y, d4.z, d4.w};
#pragma unroll
          for (int h2 = 0; h2 < 2; ++h2) {
            float pv[2], dv[2];
#pragma unroll
            for (int u = 0; u < 2; ++u) {
              const int col = 2 * (e + h2) + u;
              const int qc = c * 32 + col;
              float pp = ex2_approx(__uint_as_float(sr[col]) * sl2 - lv[2 * h2 + u]);
              if (masked && static_cast<long long>(key) > q0 + qc + p.past_len) pp = 0.f;
              pv[u] = pp;
              dv[u] = pp * (__uint_as_float(dr[col]) - dl[2 * h2 + u]);
            }
            pk[e + h2] = pack_bf16x2(pv[0], pv[1]);
            ds[e + h2] = pack_bf16x2(dv[0], dv[1]);
          }
        }
        tmem_st16(tmem + lane_base + T_ST + c * 32, pk);   // over S^T columns just read
        tmem_st16(tmem + lane_base + T_DPT + c * 32, ds);  // over dP^T columns just read
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.st_free);
        mbar_arrive(&s.pd_ready);
      }
    }
    if (ok && warp_wait(s, &s.acc_done, (n_q - 1) & 1)) {
      tc_fence_after();
      const size_t kidx = static_cast<size_t>(bh) * p.Tk + static_cast<size_t>(key);
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t acc[32];
        tmem_ld32(tmem + lane_base + T_DK + c * 32, acc);
        tmem_wait_ld();
        reg_fence(acc);
        if (key < p.Tk) store_row_bf16(p.out0 + kidx * HD + c * 32, acc, SCALE);
        tmem_ld32(tmem + lane_base + T_DV + c * 32, acc);
        tmem_wait_ld();
        reg_fence(acc);
        if (key < p.Tk) store_row_bf16(p.out1 + kidx * HD + c * 32, acc, 1.f);
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

}  // namespace backward_det
}  // namespace tt
