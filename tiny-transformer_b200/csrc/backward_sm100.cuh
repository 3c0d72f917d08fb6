// BF16 causal attention backward for sm_100a: dQ, dK, dV from q, k, v, dO, O and the forward's
// natural-log LSE. Semantics follow the reference (Tiny-transformer
// csrc/attention/attention.cu:161-234, attention_backward_preprocess_kernel.cuh,
// attention_backward_dKdV_kernel.cu, attention_backward_dQ_kernel.cu):
//   D_i   = sum_d dO[i, d] * O[i, d]                           (FP32)
//   P_ij  = exp(scale * q_i.k_j - LSE_i) on visible pairs, else 0 (FP32)
//   dS_ij = P_ij * (dO_i.v_j - D_i)                            (FP32)
//   dV_j  = sum_i bf16(P_ij) dO_i,   dK_j = scale * sum_i bf16(dS_ij) q_i,
//   dQ_i  = scale * sum_j bf16(dS_ij) k_j                      (FP32 accumulate, BF16 out)
// with key j visible to query i iff j <= i + past_len (Tk == Tq + past_len), scale = 1/8.
//
// Three kernels, in stream order:
// * bwd_preprocess_kernel: D, one warp per query row (coalesced 128-byte rows).
// * bwd_dq_kernel: one CTA per (b, h, 128-row query tile), looping over the KV tiles it sees.
//   tcgen05: S = Q.K^T and dP = dO.V^T (both SS, into TMEM), the elementwise warps (thread =
//   query row = TMEM lane) turn them into bf16 dS in TMEM, then dQ += dS.K (TS, A from TMEM).
//   TMEM: S [0,128), dP [128,256), dS [256,320), dQ [320,384).
// * bwd_dkdv_kernel: one CTA per (b, h, 128-key tile), looping over the query tiles that see
//   it, in transposed form so that keys are the TMEM lanes: S^T = K.Q^T, dP^T = V.dO^T, the
//   elementwise warps (thread = key row) write bf16 P^T and dS^T into TMEM, then
//   dV += P^T.dO and dK += dS^T.Q (TS). Per-query LSE and D come from shared memory
//   (broadcast reads). TMEM: S^T, dP^T, P^T, dS^T, dV, dK = all 512 columns.
// Roles in both: warps 0-3 elementwise + epilogue, warp 4 TMA producer (all lanes stage LSE/D
// in the dK/dV kernel), warp 5 tcgen05 issuer (one thread). Every mbarrier wait is bounded
// (TT_ERR_TIMEOUT + abort flag), as in the forward kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"
#include "prefill_sm100.cuh"

namespace tt {
namespace backward {

constexpr int BM = 128;  // query rows per tile
constexpr int BN = 128;  // keys per tile
constexpr int HD = 64;
constexpr int STAGES = 3;
constexpr int THREADS = 192;  // 4 elementwise warps, TMA warp, issuer warp
constexpr int LOAD_WARP = 4, MMA_WARP = 5;
constexpr uint32_t TILE_BYTES = 128 * HD * 2;  // 16 KiB
constexpr float SCALE = 0.125f;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.69314718055994530942f;

struct Params {
  int B, H, Tq, Tk, past_len;
  int n_tiles;              // query tiles (dQ kernel) or key tiles (dK/dV kernel)
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

__global__ void __launch_bounds__(256) bwd_preprocess_kernel(const PreParams p) {
  const long long row = static_cast<long long>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= p.rows) return;
  const uint32_t a = reinterpret_cast<const uint32_t*>(p.dO + row * HD)[lane];
  const uint32_t o = reinterpret_cast<const uint32_t*>(p.O + row * HD)[lane];
  float sum = bf16_lo(a) * bf16_lo(o) + bf16_hi(a) * bf16_hi(o);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0) p.D[row] = sum;
}

// ------------------------------------------------------------------ shared pieces
struct alignas(1024) SmemQ {  // dQ kernel
  uint8_t q[TILE_BYTES];
  uint8_t dO[TILE_BYTES];
  uint8_t k[STAGES][TILE_BYTES];
  uint8_t v[STAGES][TILE_BYTES];
  uint64_t qd_full;
  uint64_t kv_full[STAGES], kv_empty[STAGES];
  uint64_t s_full, s_free, ds_ready, dq_done, drain;
  uint32_t tmem_base;
  volatile int abort;
};

struct alignas(1024) SmemKV {  // dK/dV kernel
  uint8_t k[TILE_BYTES];
  uint8_t v[TILE_BYTES];
  uint8_t q[STAGES][TILE_BYTES];
  uint8_t dO[STAGES][TILE_BYTES];
  float lse2[STAGES][BM];  // LSE * log2(e) per query row of the stage (+inf past Tq)
  float d[STAGES][BM];
  uint64_t kv_full;
  uint64_t q_full[STAGES], q_empty[STAGES];
  uint64_t st_full, st_free, pd_ready, acc_done, drain;
  uint32_t tmem_base;
  volatile int abort;
};

constexpr size_t kSmemQ = sizeof(SmemQ) + 1024;
constexpr size_t kSmemKV = sizeof(SmemKV) + 1024;

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

// KV tiles (of BN keys) that query rows [q0, q0 + BM) see.
__device__ __forceinline__ int kv_tiles_seen(const Params& p, int q0) {
  const long long end =
      min(static_cast<long long>(p.Tk), static_cast<long long>(q0) + BM + p.past_len);
  return static_cast<int>((end + BN - 1) / BN);
}

// First query tile whose rows see key tile kt (keys [BN kt, BN kt + BN)).
__device__ __forceinline__ int first_q_tile(const Params& p, int kt) {
  const long long q_first = max(0LL, static_cast<long long>(kt) * BN - p.past_len);
  return static_cast<int>(q_first / BM);
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
__global__ void __launch_bounds__(THREADS, 1)
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
  const int q0 = qt * BM;
  const int n_kv = kv_tiles_seen(p, q0);
  constexpr uint32_t T_S = 0, T_DP = 128, T_DS = 256, T_DQ = 320;

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
    tmem_alloc(&s.tmem_base, 512);
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
        mbar_arrive_expect_tx(&s.kv_full[st], 2 * TILE_BYTES);
        tma_load_4d(s.k[st], &tm_k, &s.kv_full[st], 0, j * BN, h, b);
        tma_load_4d(s.v[st], &tm_v, &s.kv_full[st], 0, j * BN, h, b);
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
      const uint32_t idesc_s = make_idesc_bf16(BM, BN, false);
      const uint32_t idesc_o = make_idesc_bf16(BM, HD, true);
      const uint32_t q_addr = smem_u32(s.q), do_addr = smem_u32(s.dO);
      bool ok = wait_or_abort(s, &s.qd_full, 0);
      for (int j = 0; ok && j < n_kv; ++j) {
        const int st = j % STAGES;
        if (!wait_or_abort(s, &s.kv_full[st], (j / STAGES) & 1)) break;
        if (j > 0 && !wait_or_abort(s, &s.s_free, (j - 1) & 1)) break;
        tc_fence_after();
        prefill::issue_s_mma(tmem + T_S, q_addr, smem_u32(s.k[st]), idesc_s);
        prefill::issue_s_mma(tmem + T_DP, do_addr, smem_u32(s.v[st]), idesc_s);
        umma_commit(&s.s_full);
        if (!wait_or_abort(s, &s.ds_ready, j & 1)) break;
        tc_fence_after();
        prefill::issue_pv_mma(tmem + T_DQ, tmem + T_DS, smem_u32(s.k[st]), idesc_o, j > 0);
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
      if (j > 0 && !warp_wait(s, &s.dq_done, (j - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      const long long kv0 = static_cast<long long>(j) * BN;
      const bool masked = kv0 + BN - 1 > tile_limit;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld32(tmem + lane_base + T_S + c * 32, sr);
        tmem_ld32(tmem + lane_base + T_DP + c * 32, dr);
        tmem_wait_ld();
        reg_fence(sr);
        reg_fence(dr);
        uint32_t ds[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float pv[2], dv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = 2 * e + u;
            float pp = ex2_approx(__uint_as_float(sr[col]) * sl2 - lse2);
            if (masked && kv0 + c * 32 + col > row_limit) pp = 0.f;
            pv[u] = pp;
            dv[u] = pp * (__uint_as_float(dr[col]) - drow);
          }
          ds[e] = pack_bf16x2(dv[0], dv[1]);
        }
        tmem_st16(tmem + lane_base + T_DS + c * 16, ds);
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
    tmem_dealloc(tmem, 512);
  }
}

// ------------------------------------------------------------------ dK/dV kernel
__global__ void __launch_bounds__(THREADS, 1)
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
  const int k0 = kt * BN;
  const int qt0 = first_q_tile(p, kt);
  const int n_q = (p.Tq + BM - 1) / BM - qt0;  // >= 1: the last query row sees every key
  constexpr uint32_t T_ST = 0, T_DPT = 128, T_PT = 256, T_DST = 320, T_DV = 384, T_DK = 448;

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
    tmem_alloc(&s.tmem_base, 512);
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
      const int q0 = (qt0 + i) * BM;
      if (i >= STAGES && !warp_wait(s, &s.q_empty[st], ((i / STAGES) - 1) & 1)) break;
      // Per-query LSE (log2 units) and D of this tile; rows past Tq get +inf / 0, so their
      // probabilities are exactly zero.
#pragma unroll
      for (int e = 0; e < BM / 32; ++e) {
        const int rr = e * 32 + lane;
        const int q = q0 + rr;
        const size_t idx = static_cast<size_t>(bh) * p.Tq + static_cast<size_t>(q);
        s.lse2[st][rr] = q < p.Tq ? p.lse[idx] * LOG2E : INFINITY;
        s.d[st][rr] = q < p.Tq ? p.D[idx] : 0.f;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(&s.q_full[st], 2 * TILE_BYTES);
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
      const uint32_t idesc_s = make_idesc_bf16(BN, BM, false);
      const uint32_t idesc_o = make_idesc_bf16(BN, HD, true);
      const uint32_t k_addr = smem_u32(s.k), v_addr = smem_u32(s.v);
      bool ok = wait_or_abort(s, &s.kv_full, 0);
      for (int i = 0; ok && i < n_q; ++i) {
        const int st = i % STAGES;
        if (!wait_or_abort(s, &s.q_full[st], (i / STAGES) & 1)) break;
        if (i > 0 && !wait_or_abort(s, &s.st_free, (i - 1) & 1)) break;
        tc_fence_after();
        prefill::issue_s_mma(tmem + T_ST, k_addr, smem_u32(s.q[st]), idesc_s);
        prefill::issue_s_mma(tmem + T_DPT, v_addr, smem_u32(s.dO[st]), idesc_s);
        umma_commit(&s.st_full);
        if (!wait_or_abort(s, &s.pd_ready, i & 1)) break;
        tc_fence_after();
        prefill::issue_pv_mma(tmem + T_DV, tmem + T_PT, smem_u32(s.dO[st]), idesc_o, i > 0);
        prefill::issue_pv_mma(tmem + T_DK, tmem + T_DST, smem_u32(s.q[st]), idesc_o, i > 0);
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
      const long long q0 = static_cast<long long>(qt0 + i) * BM;
      if (!warp_wait(s, &s.st_full, i & 1)) { ok = false; break; }
      if (i > 0 && !warp_wait(s, &s.acc_done, (i - 1) & 1)) { ok = false; break; }
      tc_fence_after();
      // Pair (key, q) is visible iff key <= q + past_len; only tiles crossing the diagonal mask.
      const bool masked = static_cast<long long>(k0) + BN - 1 > q0 + p.past_len;
#pragma unroll 1
      for (int c = 0; c < BM / 32; ++c) {
        uint32_t sr[32], dr[32];
        tmem_ld32(tmem + lane_base + T_ST + c * 32, sr);
        tmem_ld32(tmem + lane_base + T_DPT + c * 32, dr);
        tmem_wait_ld();
        reg_fence(sr);
        reg_fence(dr);
        uint32_t pk[16], ds[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          float pv[2], dv[2];
#pragma unroll
          for (int u = 0; u < 2; ++u) {
            const int col = 2 * e + u;
            const int qc = c * 32 + col;
            float pp = ex2_approx(__uint_as_float(sr[col]) * sl2 - s.lse2[st][qc]);
            if (masked && static_cast<long long>(key) > q0 + qc + p.past_len) pp = 0.f;
            pv[u] = pp;
            dv[u] = pp * (__uint_as_float(dr[col]) - s.d[st][qc]);
          }
          pk[e] = pack_bf16x2(pv[0], pv[1]);
          ds[e] = pack_bf16x2(dv[0], dv[1]);
        }
        tmem_st16(tmem + lane_base + T_PT + c * 16, pk);
        tmem_st16(tmem + lane_base + T_DST + c * 16, ds);
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
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace backward
}  // namespace tt
