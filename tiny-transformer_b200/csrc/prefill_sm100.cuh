// BF16 causal attention forward (prefill / chunked prefill) for sm_100a.
//
// Semantics follow the reference operator (tiny_transformer/operators/reference.py:37-53 and
// csrc/attention/attention_forward_BF16_kernel.cuh:232-389 in Tiny-transformer):
//   key j is visible to query row i iff j <= i + past_len (inclusive causal, Tk == past_len + Tq),
//   softmax scale 1/sqrt(64), FP32 softmax, P rounded to BF16 before P.V,
//   O in BF16, LSE = natural-log logsumexp of the scaled scores in FP32.
//
// One CTA computes one 128-row query tile of one (batch, head). Roles (6 warps):
//   warps 0-3  softmax + epilogue: thread t owns query row t of the tile (TMEM lane t)
//   warp  4    TMA producer: Q tile once, then K/V tiles through a STAGES-deep ring
//   warp  5    tcgen05 issuer: S = Q.K^T (SS form) and O += P.V (TS form, P read from TMEM)
// TMEM (256 columns): S in [0,128), P (bf16x2) in [128,192), O in [192,256).
// Two CTAs fit on one SM (TMEM 2 x 256 columns, ~82 KB shared memory each), so one
// CTA's softmax overlaps the other CTA's tensor-core work.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace tt {
namespace prefill {

constexpr int BM = 128;                 // query rows per tile (UMMA M)
constexpr int BN = 128;                 // keys per KV tile (UMMA N of S)
constexpr int HD = 64;                  // head dim
constexpr int STAGES = 2;               // K/V ring depth
constexpr int THREADS = 192;
constexpr int LOAD_WARP = 4;
constexpr int MMA_WARP = 5;
constexpr uint32_t TILE_BYTES = BM * HD * 2;  // 16 KiB, one 128x64 bf16 tile
constexpr uint32_t TMEM_COLS = 256;
constexpr uint32_t S_COL = 0, P_COL = 128, O_COL = 192;
constexpr float LN2 = 0.69314718055994530942f;
// O is rescaled only when the running row max grows by more than this (log2 units);
// between rescales P stays below 2^8, far inside the FP32/BF16 range.
constexpr float RESCALE_THRESHOLD = 8.0f;

struct alignas(1024) Smem {
  uint8_t q[TILE_BYTES];
  uint8_t k[STAGES][TILE_BYTES];
  uint8_t v[STAGES][TILE_BYTES];
  uint64_t q_full;
  uint64_t k_full[STAGES], k_empty[STAGES];
  uint64_t v_full[STAGES], v_empty[STAGES];
  uint64_t s_full, s_free, p_ready, pv_done, drain;
  uint32_t tmem_base;
  volatile int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack for 1 KiB alignment

struct Params {
  int B, H, Tq, Tk, past_len;
  int n_qtiles;
  __nv_bfloat16* o;  // contiguous [B, H, Tq, 64]
  float* lse;        // contiguous [B, H, Tq]
  float scale_log2;  // softmax scale * log2(e)
};

// Bounded wait that also gives up as soon as another role has aborted.
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

// Warp-uniform wait: every lane waits, and the warp proceeds only if all lanes saw
// the phase complete (lanes can disagree only when the CTA is aborting).
__device__ __forceinline__ bool warp_wait(Smem& s, uint64_t* bar, uint32_t parity) {
  const bool ok = wait_or_abort(s, bar, parity);
  return __all_sync(0xffffffffu, ok);
}

__device__ __forceinline__ void issue_s_mma(uint32_t tmem_s, uint32_t q_addr, uint32_t k_addr,
                                            uint32_t idesc) {
  // K = 64 features = 4 UMMA k-steps of 16; each step advances 32 bytes inside the
  // 128-byte swizzled row. SBO = 1024 B between 8-row swizzle atoms.
#pragma unroll
  for (int kk = 0; kk < HD / 16; ++kk) {
    const uint64_t a = make_sdesc_sw128(q_addr + kk * 32, 16, 1024);
    const uint64_t b = make_sdesc_sw128(k_addr + kk * 32, 16, 1024);
    umma_ss(tmem_s, a, b, idesc, kk > 0 ? 1u : 0u);
  }
}

__device__ __forceinline__ void issue_pv_mma(uint32_t tmem_o, uint32_t tmem_p, uint32_t v_addr,
                                             uint32_t idesc, bool accumulate) {
  // K = 128 keys = 8 k-steps of 16 keys. P: 8 TMEM columns per step (bf16x2).
  // V is the MN-major B operand: 16 key rows x 128 B = 2048 B per step, SBO = 1024 B.
#pragma unroll
  for (int kk = 0; kk < BN / 16; ++kk) {
    const uint64_t b = make_sdesc_sw128(v_addr + kk * 2048, 8192, 1024);
    umma_ts(tmem_o, tmem_p + kk * 8, b, idesc, (accumulate || kk > 0) ? 1u : 0u);
  }
}

__global__ void __launch_bounds__(THREADS, 2)
attention_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Heaviest causal tiles first: blocks are dispatched roughly in index order.
  const int BH = p.B * p.H;
  const int qt = p.n_qtiles - 1 - static_cast<int>(blockIdx.x / BH);
  const int bh = static_cast<int>(blockIdx.x % BH);
  const int b = bh / p.H;
  const int h = bh % p.H;
  const int q0 = qt * BM;
  const long long kv_end_ll =
      min(static_cast<long long>(p.Tk), static_cast<long long>(q0) + BM + p.past_len);
  const int n_kv = static_cast<int>((kv_end_ll + BN - 1) / BN);

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], 1);
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], 1);
    }
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_free, 4);
    mbar_init(&s.p_ready, 4);
    mbar_init(&s.pv_done, 1);
    mbar_init(&s.drain, 1);
    s.abort = 0;
    fence_barrier_init();
  }
  if (warp == MMA_WARP) {
    tmem_alloc(&s.tmem_base, TMEM_COLS);
    tmem_relinquish();
  }
  if (warp == LOAD_WARP && lane == 0) {
    tma_prefetch_desc(&tm_q);
    tma_prefetch_desc(&tm_k);
    tma_prefetch_desc(&tm_v);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s.tmem_base;

  if (warp == LOAD_WARP) {
    if (lane == 0) {
      int issued_k = 0, issued_v = 0;  // K / V tiles whose loads were issued
      mbar_arrive_expect_tx(&s.q_full, TILE_BYTES);
      tma_load_4d(s.q, &tm_q, &s.q_full, 0, q0, h, b);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % STAGES;
        const uint32_t use = j / STAGES;
        if (j >= STAGES && !wait_or_abort(s, &s.k_empty[st], (use - 1) & 1)) break;
        mbar_arrive_expect_tx(&s.k_full[st], TILE_BYTES);
        tma_load_4d(s.k[st], &tm_k, &s.k_full[st], 0, j * BN, h, b);
        issued_k = j + 1;
        if (j >= STAGES && !wait_or_abort(s, &s.v_empty[st], (use - 1) & 1)) break;
        mbar_arrive_expect_tx(&s.v_full[st], TILE_BYTES);
        tma_load_4d(s.v[st], &tm_v, &s.v_full[st], 0, j * BN, h, b);
        issued_v = j + 1;
      }
      if (s.abort) {
        // Drain: never leave the CTA while a TMA write into its shared memory is pending.
        mbar_wait(&s.q_full, 0);
        for (int j = max(0, issued_k - STAGES); j < issued_k; ++j)
          mbar_wait(&s.k_full[j % STAGES], (j / STAGES) & 1);
        for (int j = max(0, issued_v - STAGES); j < issued_v; ++j)
          mbar_wait(&s.v_full[j % STAGES], (j / STAGES) & 1);
      }
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(BM, BN, false);
      const uint32_t idesc_o = make_idesc_bf16(BM, HD, true);
      const uint32_t q_addr = smem_u32(s.q);
      bool ok = wait_or_abort(s, &s.q_full, 0) && wait_or_abort(s, &s.k_full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_s_mma(tmem + S_COL, q_addr, smem_u32(s.k[0]), idesc_s);
        umma_commit(&s.s_full);
        umma_commit(&s.k_empty[0]);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j + 1 < n_kv) {
          const int st1 = (j + 1) % STAGES;
          if (!wait_or_abort(s, &s.k_full[st1], ((j + 1) / STAGES) & 1)) break;
          if (!wait_or_abort(s, &s.s_free, j & 1)) break;
          tc_fence_after();
          issue_s_mma(tmem + S_COL, q_addr, smem_u32(s.k[st1]), idesc_s);
          umma_commit(&s.s_full);
          umma_commit(&s.k_empty[st1]);
        }
        const int st = j % STAGES;
        if (!wait_or_abort(s, &s.p_ready, j & 1)) break;
        if (!wait_or_abort(s, &s.v_full[st], (j / STAGES) & 1)) break;
        tc_fence_after();
        issue_pv_mma(tmem + O_COL, tmem + P_COL, smem_u32(s.v[st]), idesc_o, j > 0);
        umma_commit(&s.pv_done);
        umma_commit(&s.v_empty[st]);
      }
      // All MMAs issued by this thread have completed once `drain` flips.
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0);
    }
  } else {
    // ---------------------------------------------------------------- softmax warps
    const int r = warp * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t t_s = tmem + lane_base + S_COL;
    const uint32_t t_p = tmem + lane_base + P_COL;
    const uint32_t t_o = tmem + lane_base + O_COL;
    const long long row_limit = static_cast<long long>(q0) + r + p.past_len;  // last visible key
    const long long tile_limit = static_cast<long long>(q0) + p.past_len;     // row 0's limit
    const float sl2 = p.scale_log2;
    float m_run = -INFINITY;  // running max of scaled scores, log2 units
    float l_run = 0.f;        // running sum of exp2(x - m_run)
    bool ok = true;

    for (int j = 0; j < n_kv; ++j) {
      if (!warp_wait(s, &s.s_full, j & 1)) { ok = false; break; }
      tc_fence_after();
      float x[BN];
      {
        uint32_t raw[BN / 32][32];
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) tmem_ld32(t_s + c * 32, raw[c]);
        tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < BN / 32; ++c) {
          reg_fence(raw[c]);
#pragma unroll
          for (int i = 0; i < 32; ++i) x[c * 32 + i] = __uint_as_float(raw[c][i]);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.s_free);

      const long long kv0 = static_cast<long long>(j) * BN;
      if (kv0 + BN - 1 > tile_limit) {
#pragma unroll
        for (int c = 0; c < BN; ++c)
          if (kv0 + c > row_limit) x[c] = -INFINITY;
      }
      float mx = x[0];
#pragma unroll
      for (int c = 1; c < BN; ++c) mx = fmaxf(mx, x[c]);
      const float m_new = fmaxf(m_run, mx * sl2);
      bool need = false;
      float factor = 1.f;
      if (j == 0) {
        m_run = m_new;
      } else if (m_new > m_run + RESCALE_THRESHOLD) {
        need = true;
        factor = ex2_approx(m_run - m_new);
        m_run = m_new;
      }
      const float m_use = (m_run == -INFINITY) ? 0.f : m_run;
      uint32_t pk[BN / 2];
      float rowsum = 0.f;
#pragma unroll
      for (int c = 0; c < BN / 2; ++c) {
        const float p0 = ex2_approx(fmaf(x[2 * c], sl2, -m_use));
        const float p1 = ex2_approx(fmaf(x[2 * c + 1], sl2, -m_use));
        rowsum += p0 + p1;
        pk[c] = pack_bf16x2(p0, p1);
      }
      l_run = l_run * factor + rowsum;

      if (j > 0) {
        // P and O are still in use by P.V of the previous tile until pv_done flips.
        if (!warp_wait(s, &s.pv_done, (j - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        if (__any_sync(0xffffffffu, need)) {
          uint32_t o[HD / 32][32];
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) tmem_ld32(t_o + c * 32, o[c]);
          tmem_wait_ld();
#pragma unroll
          for (int c = 0; c < HD / 32; ++c) {
            reg_fence(o[c]);
#pragma unroll
            for (int i = 0; i < 32; ++i)
              o[c][i] = __float_as_uint(__uint_as_float(o[c][i]) * factor);
            tmem_st32(t_o + c * 32, o[c]);
          }
        }
      }
      {
        uint32_t half[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) half[i] = pk[i];
        tmem_st32(t_p, half);
#pragma unroll
        for (int i = 0; i < 32; ++i) half[i] = pk[32 + i];
        tmem_st32(t_p + 32, half);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_ready);
    }

    if (ok && warp_wait(s, &s.pv_done, (n_kv - 1) & 1)) {
      tc_fence_after();
      const int row = q0 + r;
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      uint32_t o[HD / 32][32];
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) tmem_ld32(t_o + c * 32, o[c]);
      tmem_wait_ld();
      if (row < p.Tq) {
        __nv_bfloat16* orow =
            p.o + (static_cast<size_t>(bh) * p.Tq + static_cast<size_t>(row)) * HD;
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          reg_fence(o[c]);
          uint32_t packed[16];
#pragma unroll
          for (int i = 0; i < 16; ++i)
            packed[i] = pack_bf16x2(__uint_as_float(o[c][2 * i]) * inv_l,
                                    __uint_as_float(o[c][2 * i + 1]) * inv_l);
          uint4* dst = reinterpret_cast<uint4*>(orow + c * 32);
#pragma unroll
          for (int i = 0; i < 4; ++i)
            dst[i] = make_uint4(packed[4 * i], packed[4 * i + 1], packed[4 * i + 2],
                                packed[4 * i + 3]);
        }
        p.lse[static_cast<size_t>(bh) * p.Tq + row] =
            l_run > 0.f ? (m_run + log2f(l_run)) * LN2 : -INFINITY;
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

}  // namespace prefill
}  // namespace tt
