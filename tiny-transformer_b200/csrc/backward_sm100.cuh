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
// * bwd_preprocess_kernel: -D and -LSE * log2(e) per query row, in rows padded to whole
//   128-row tiles (eight lanes per row, 16-byte loads of dO and O), and zeros for the row's
//   FP32 dQ accumulator (the same pass instead of a separate memset), plus the work counter of
//   the persistent kernel.
// * persist::bwd_persistent_kernel (default): one CTA per SM running (b, h, 128-key tile) items
//   back to back, or fused::bwd_fused_kernel: one CTA per item. Either way S, dP and the
//   exponentials are computed once per (query tile, key tile) pair and feed dV, dK and dQ.
// * fused::bwd_dq_convert_kernel: dQ = bf16(scale * dQ accumulator).
// Every mbarrier wait is bounded (TT_ERR_TIMEOUT + abort flag), as in the forward kernels.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace tt {
namespace backward {

constexpr int HD = 64;
constexpr float SCALE = 0.125f;
constexpr float LOG2E = 1.4426950408889634f;

// ------------------------------------------------------------------ preprocess
struct PreParams {
  long long rows;            // B * H * Tq_pad (query rows padded to whole 128-row tiles)
  int Tq, Tq_pad;
  const __nv_bfloat16* dO;   // contiguous [B * H * Tq, 64]
  const __nv_bfloat16* O;
  const float* lse;          // contiguous [B * H * Tq], natural log
  float* nlse2;              // [B * H * Tq_pad]: -LSE * log2(e), -inf on padding rows
  float* nd;                 // [B * H * Tq_pad]: -D, 0 on padding rows
  float* dq_acc;             // [B * H * Tq, 64]: set to zero
  unsigned int* next_item;   // work counter of bwd_persistent_kernel: set to zero
};

// Eight lanes per row, 16-byte loads: a warp covers four rows, a block of 256 threads 32.
constexpr int PRE_ROWS_PER_BLOCK = 32;

__global__ void __launch_bounds__(256) bwd_preprocess_kernel(const PreParams p) {
  const long long prow =
      static_cast<long long>(blockIdx.x) * PRE_ROWS_PER_BLOCK + (threadIdx.x >> 3);
  const int part = threadIdx.x & 7;  // 8 features per lane
  const long long bh = prow / p.Tq_pad;
  const int q = static_cast<int>(prow - bh * p.Tq_pad);
  const bool real = prow < p.rows && q < p.Tq;
  if (prow == 0 && part == 0) *p.next_item = 0u;
  const long long row = bh * p.Tq + q;
  float sum = 0.f;
  if (real) {
    const uint4 a = reinterpret_cast<const uint4*>(p.dO + row * HD)[part];
    const uint4 o = reinterpret_cast<const uint4*>(p.O + row * HD)[part];
    sum = bf16_lo(a.x) * bf16_lo(o.x) + bf16_hi(a.x) * bf16_hi(o.x) +
          bf16_lo(a.y) * bf16_lo(o.y) + bf16_hi(a.y) * bf16_hi(o.y) +
          bf16_lo(a.z) * bf16_lo(o.z) + bf16_hi(a.z) * bf16_hi(o.z) +
          bf16_lo(a.w) * bf16_lo(o.w) + bf16_hi(a.w) * bf16_hi(o.w);
    float4* acc = reinterpret_cast<float4*>(p.dq_acc + row * HD) + 2 * part;
    acc[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    acc[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // Reduce over the eight lanes of the row (all 32 lanes take part in every shuffle).
#pragma unroll
  for (int off = 4; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (part == 0 && prow < p.rows) {
    p.nd[prow] = real ? -sum : 0.f;
    p.nlse2[prow] = real ? -p.lse[row] * LOG2E : -INFINITY;
  }
}

// ------------------------------------------------------------------ shared pieces
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

// ------------------------------------------------------------------ fused dQ/dK/dV kernel
// One CTA per (b, h, 128-key tile), stepping over 128-row query tiles in transposed form (keys
// are the TMEM lanes). Per step, all products are M = 128 tcgen05 MMAs:
//   S^T = K.Q^T, dP^T = V.dO^T        (SS, N = 128)
//   dV += P^T.dO                      (TS, A = bf16 P^T in its own TMEM columns)
//   dK += dS^T.Q                      (SS, A = the shared-memory dS tile read K-major)
//   dQ_step = dS.K                    (SS, A = the same dS tile read MN-major)
// dQ_step is read out of TMEM by four drain warps and added into an FP32 dQ workspace with TMA
// bulk reduce-add (32 x 32 boxes, the two feature halves of a warp's rows one after the other
// through one staging box); bwd_dq_convert_kernel scales it
// and rounds it to bf16 afterwards. S, dP and the exponentials are computed once per pair of
// tiles, and every score product has N = 128.
//
// The elementwise warps work in two phases per step: (1) load S^T, release it, compute
// P = exp2(S * scale * log2(e) - LSE * log2(e)) and store bf16 P^T; (2) load dP^T, compute
// dS = P * (dP - D) from the FP32 P kept in registers, store bf16 dS into shared memory.
// Two issuer threads feed the tensor core (a tcgen05.mma blocks its thread for
// about its execution time, so one thread would delay each product behind the others):
//   scores issuer:     S^T(i+1) once S^T(i) is released (overlapping both phases of step i);
//                      dP^T(i+1) once the elementwise warps have read dP^T(i);
//   accumulate issuer: dV(i) once P^T(i) is stored; dK(i), then dQ(i), once dS(i) is stored;
// so phase 1 of step i+1 starts as soon as phase 2 of step i ends. (Measured on cfg3 against
// other assignments: S and dV on one thread with dK, dP, dQ on the other, 5 % slower; three
// issuer warps, 2-5 % slower.)
// TMEM: S^T [0,128), dP^T [128,256), dV [256,320), dK [320,384), dQ [384,448),
// P^T [448,512) of 512 columns.
// Roles: warps 0-7 elementwise (warp w: TMEM lanes 32 (w % 4) .., query columns 64 (w / 4) ..),
// warps 8-11 dQ drain (lanes 32 (w % 4) ..), warp 12 TMA producer, warp 13 accumulate issuer
// (and TMEM owner), warp 14 scores issuer.
namespace fused {

constexpr int T = 128;          // keys per CTA tile and query rows per step
constexpr int STAGES = 3;       // Q / dO / LSE / D ring
constexpr int EW_WARPS = 8, DQ_WARP0 = 8, LOAD_WARP = 12, MMA_WARP = 13, SCORE_WARP = 14;
constexpr int THREADS = 15 * 32;
constexpr uint32_t TILE_BYTES = T * HD * 2;  // 16 KiB
constexpr uint32_t T_ST = 0, T_DPT = 128, T_DV = 256, T_DK = 320, T_DQ = 384, T_P = 448;
constexpr uint32_t TMEM_COLS = 512;
constexpr int DQ_BOX_ROWS = 32;  // dQ reduce box: 32 rows x 32 FP32 features (128 B, SW128)

struct Params {
  int B, H, Tq, Tk, past_len;
  int n_k_tiles;
  int Tq_pad;           // Tq rounded up to whole 128-row tiles
  const float* nlse2;   // [B, H, Tq_pad]: -LSE * log2(e), -inf on padding rows
  const float* nd;      // [B, H, Tq_pad]: -D
  __nv_bfloat16* dk;    // contiguous [B, H, Tk, 64]
  __nv_bfloat16* dv;
};

struct alignas(1024) Smem {
  uint8_t k[TILE_BYTES];
  uint8_t v[TILE_BYTES];
  uint8_t q[STAGES][TILE_BYTES];
  uint8_t dO[STAGES][TILE_BYTES];
  // dS of the step as the MN-major A operand of dQ = dS.K: atom column c (queries [64c, 64c+64))
  // holds one 128-byte row per key (K index), 16-byte chunks XOR-swizzled by key & 7.
  uint8_t ds[2][T * 128];
  // Per drain warp, one feature half of its 32 dQ rows at a time, 128-byte swizzled.
  uint8_t dq_stage[4][DQ_BOX_ROWS * 128];
  float nlse2[STAGES][T];  // -LSE * log2(e) per query row of the stage (-inf past Tq)
  float nd[STAGES][T];     // -D per query row of the stage
  uint64_t kv_full;
  uint64_t q_full[STAGES], q_empty[STAGES];
  uint64_t s_full, s_consumed, p_full, pv_free, dp_full, ds_ready, ds_free;
  uint64_t dq_full, dq_free, acc_final, drain, drain_scores;
  uint32_t tmem_base;
  volatile int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 227 * 1024, "fused backward shared memory");

// dQ_step = dS.K: A = dS (MN-major, two 64-query atom columns 16 KiB apart), B = K tile
// (MN-major over features), K = 128 keys in 8 steps of 16 key rows (2048 B in both operands).
__device__ __forceinline__ void issue_dq(uint32_t tmem_d, uint32_t ds_addr, uint32_t k_addr,
                                         uint32_t idesc) {
#pragma unroll
  for (int kk = 0; kk < T / 16; ++kk)
    umma_ss(tmem_d, make_sdesc_sw128(ds_addr + kk * 2048, T * 128, 1024),
            make_sdesc_sw128(k_addr + kk * 2048, 8192, 1024), idesc, kk > 0 ? 1u : 0u);
}

// dV += P^T.dO: A = bf16 P^T pairs in TMEM (8 columns per k-step), B = dO (MN-major over
// features), K = 128 queries in 8 steps of 16 rows (2048 B per step).
__device__ __forceinline__ void issue_dv(uint32_t tmem_d, uint32_t tmem_a, uint32_t b_addr,
                                         uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < T / 16; ++kk)
    umma_ts(tmem_d, tmem_a + 8 * kk, make_sdesc_sw128(b_addr + kk * 2048, 8192, 1024), idesc,
            (accumulate || kk > 0) ? 1u : 0u);
}

// dK += dS^T.Q: A = the shared-memory dS tile read as a K-major operand (row = key, 64 queries
// of one atom column per 128-byte row, so k-step kk is 32 bytes into atom column kk / 4),
// B = Q (MN-major over features, 2048 B per 16-query step). Reading dS from shared memory
// leaves the dP^T columns free for the next step's dP^T as soon as the elementwise warps have
// read them, instead of after dK.
__device__ __forceinline__ void issue_dk(uint32_t tmem_d, uint32_t ds_addr, uint32_t q_addr,
                                         uint32_t idesc, bool accumulate) {
#pragma unroll
  for (int kk = 0; kk < T / 16; ++kk)
    umma_ss(tmem_d, make_sdesc_sw128(ds_addr + (kk >> 2) * (T * 128) + (kk & 3) * 32, 16, 1024),
            make_sdesc_sw128(q_addr + kk * 2048, 8192, 1024), idesc,
            (accumulate || kk > 0) ? 1u : 0u);
}

// Phase 1 for one 32-query chunk: p = exp2(S * scale * log2(e) - LSE * log2(e)), packed to bf16
// pairs; with MASKED, queries before chunk column `first_visible` get p = 0.
template <bool MASKED>
__device__ __forceinline__ void ew_probs(const uint32_t (&sr)[32], uint32_t nlse_addr,
                                         int first_visible, float* p, uint32_t (&pk)[16]) {
  const uint64_t sc2 = f2_pack(SCALE * LOG2E, SCALE * LOG2E);
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const float4 nl = lds_f4(nlse_addr + 16 * g);
    float x[4];
    f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[4 * g]), __uint_as_float(sr[4 * g + 1])), sc2,
                     f2_pack(nl.x, nl.y)), x[0], x[1]);
    f2_unpack(f2_fma(f2_pack(__uint_as_float(sr[4 * g + 2]), __uint_as_float(sr[4 * g + 3])), sc2,
                     f2_pack(nl.z, nl.w)), x[2], x[3]);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      p[4 * g + u] = ex2_approx(x[u]);
      if (MASKED && 4 * g + u < first_visible) p[4 * g + u] = 0.f;
    }
    pk[2 * g] = pack_bf16x2(p[4 * g], p[4 * g + 1]);
    pk[2 * g + 1] = pack_bf16x2(p[4 * g + 2], p[4 * g + 3]);
  }
}

// Phase 2 for 16 queries: ds = p * (dP - D), packed to bf16 pairs (p: the 16 FP32
// probabilities of these queries).
__device__ __forceinline__ void ew_dscores(const float* p, const uint32_t (&dr)[16],
                                           uint32_t nd_addr, uint32_t (&dsb)[8]) {
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    const float4 nd = lds_f4(nd_addr + 16 * g);
    const uint64_t d01 = f2_add(
        f2_pack(__uint_as_float(dr[4 * g]), __uint_as_float(dr[4 * g + 1])), f2_pack(nd.x, nd.y));
    const uint64_t d23 = f2_add(
        f2_pack(__uint_as_float(dr[4 * g + 2]), __uint_as_float(dr[4 * g + 3])), f2_pack(nd.z, nd.w));
    float ds[4];
    f2_unpack(f2_mul(f2_pack(p[4 * g], p[4 * g + 1]), d01), ds[0], ds[1]);
    f2_unpack(f2_mul(f2_pack(p[4 * g + 2], p[4 * g + 3]), d23), ds[2], ds[3]);
    dsb[2 * g] = pack_bf16x2(ds[0], ds[1]);
    dsb[2 * g + 1] = pack_bf16x2(ds[2], ds[3]);
  }
}

__global__ void __launch_bounds__(THREADS, 1)
bwd_fused_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                 const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                 const __grid_constant__ CUtensorMap tm_dqacc, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int BH = p.B * p.H;
  const int kt = static_cast<int>(blockIdx.x / BH);  // low key tiles see the most queries
  const int bh = static_cast<int>(blockIdx.x % BH);
  const int b = bh / p.H, h = bh % p.H;
  const int k0 = kt * T;
  // Query tiles that see some key of this tile: from the one holding query k0 - past_len on.
  const int qt0 = static_cast<int>(max(0LL, static_cast<long long>(k0) - p.past_len) / T);
  const int n_q = (p.Tq + T - 1) / T - qt0;

  if (threadIdx.x == 0) {
    mbar_init(&s.kv_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 1);
    }
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_consumed, EW_WARPS);
    mbar_init(&s.p_full, EW_WARPS);
    mbar_init(&s.pv_free, 1);
    mbar_init(&s.dp_full, 1);
    mbar_init(&s.ds_ready, EW_WARPS);
    mbar_init(&s.ds_free, 1);
    mbar_init(&s.dq_full, 1);
    mbar_init(&s.dq_free, 4);
    mbar_init(&s.acc_final, 1);
    mbar_init(&s.drain, 1);
    mbar_init(&s.drain_scores, 1);
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
      const int q0 = (qt0 + i) * T;
      if (i >= STAGES && !warp_wait(s, &s.q_empty[st], ((i / STAGES) - 1) & 1)) break;
      if (lane == 0) {
        const size_t row = static_cast<size_t>(bh) * p.Tq_pad + static_cast<size_t>(q0);
        mbar_arrive_expect_tx(&s.q_full[st], 2 * TILE_BYTES + 2 * T * sizeof(float));
        tma_load_4d(s.q[st], &tm_q, &s.q_full[st], 0, q0, h, b);
        tma_load_4d(s.dO[st], &tm_do, &s.q_full[st], 0, q0, h, b);
        bulk_load_plain(s.nlse2[st], p.nlse2 + row, T * sizeof(float), &s.q_full[st]);
        bulk_load_plain(s.nd[st], p.nd + row, T * sizeof(float), &s.q_full[st]);
      }
      issued = i + 1;
    }
    if (lane == 0 && s.abort) {
      mbar_wait(&s.kv_full, 0);
      for (int i = max(0, issued - STAGES); i < issued; ++i)
        mbar_wait(&s.q_full[i % STAGES], (i / STAGES) & 1);
    }
  } else if (warp == SCORE_WARP) {
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(T, T, false);
      const uint32_t k_addr = smem_u32(s.k), v_addr = smem_u32(s.v);
      bool ok = wait_or_abort(s, &s.kv_full, 0) && wait_or_abort(s, &s.q_full[0], 0);
      if (ok) {
        tc_fence_after();
        issue_scores(tmem + T_ST, k_addr, smem_u32(s.q[0]), idesc_s);
        umma_commit(&s.s_full);
        issue_scores(tmem + T_DPT, v_addr, smem_u32(s.dO[0]), idesc_s);
        umma_commit(&s.dp_full);
      }
      for (int i = 0; ok && i + 1 < n_q; ++i) {
        const int sn = (i + 1) % STAGES;
        if (!wait_or_abort(s, &s.q_full[sn], ((i + 1) / STAGES) & 1)) break;
        // S^T(i+1) as soon as the elementwise warps hold S^T(i) in registers.
        if (!wait_or_abort(s, &s.s_consumed, i & 1)) break;
        tc_fence_after();
        issue_scores(tmem + T_ST, k_addr, smem_u32(s.q[sn]), idesc_s);
        umma_commit(&s.s_full);
        // dP^T(i+1) overwrites dP^T(i): once the elementwise warps have read it.
        if (!wait_or_abort(s, &s.ds_ready, i & 1)) break;
        tc_fence_after();
        issue_scores(tmem + T_DPT, v_addr, smem_u32(s.dO[sn]), idesc_s);
        umma_commit(&s.dp_full);
      }
      umma_commit(&s.drain_scores);
      mbar_wait(&s.drain_scores, 0);
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc_o = make_idesc_bf16(T, HD, true);
      const uint32_t idesc_dq = make_idesc_bf16(T, HD, true) | (1u << 15);  // A MN-major
      const uint32_t k_addr = smem_u32(s.k);
      for (int i = 0; i < n_q; ++i) {
        const int st = i % STAGES;
        if (!wait_or_abort(s, &s.p_full, i & 1)) break;
        tc_fence_after();
        issue_dv(tmem + T_DV, tmem + T_P, smem_u32(s.dO[st]), idesc_o, i > 0);
        umma_commit(&s.pv_free);
        if (!wait_or_abort(s, &s.ds_ready, i & 1)) break;
        tc_fence_after();
        issue_dk(tmem + T_DK, smem_u32(s.ds[0]), smem_u32(s.q[st]), idesc_o, i > 0);
        // Q(i) and dO(i) were last read by dV(i) and dK(i); S^T(i) and dP^T(i) (scores
        // issuer) completed before the elementwise warps could read them.
        umma_commit(&s.q_empty[st]);
        if (i + 1 == n_q) umma_commit(&s.acc_final);
        if (i > 0 && !wait_or_abort(s, &s.dq_free, (i - 1) & 1)) break;
        tc_fence_after();
        issue_dq(tmem + T_DQ, smem_u32(s.ds[0]), k_addr, idesc_dq);
        umma_commit(&s.dq_full);
        umma_commit(&s.ds_free);
      }
      // All MMAs issued by this thread have completed once `drain` flips.
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0);
    }
  } else if (warp >= DQ_WARP0 && warp < DQ_WARP0 + 4) {
    // dQ drain: thread = query row 32 * quarter + lane of the step = TMEM lane.
    const int quarter = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* box = s.dq_stage[quarter];
    for (int i = 0; i < n_q; ++i) {
      if (!warp_wait(s, &s.dq_full, i & 1)) break;
      tc_fence_after();
      uint32_t a0[32], a1[32];
      tmem_ld32(tmem + lane_base + T_DQ, a0);
      tmem_ld32(tmem + lane_base + T_DQ + 32, a1);
      tmem_wait_ld();
      reg_fence(a0);
      reg_fence(a1);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(&s.dq_free);
        bulk_wait_group_read_all();  // the previous step's reduce has read the staging boxes
      }
      __syncwarp();
      const uint32_t sw = lane & 7;
      const uint32_t row_addr = smem_u32(box) + lane * 128;
      const int row0 = (qt0 + i) * T + quarter * DQ_BOX_ROWS;
      // One staging box per warp: features [0, 32), then [32, 64) once the first reduce has
      // read the box.
#pragma unroll
      for (uint32_t j = 0; j < 8; ++j)
        sts_u4(row_addr + ((j ^ sw) << 4), a0[4 * j], a0[4 * j + 1], a0[4 * j + 2], a0[4 * j + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 < p.Tq) {  // rows past Tq inside a box are clipped by the map
        tma_reduce_add_4d(box, &tm_dqacc, 0, row0, h, b);
        bulk_commit_group();
        bulk_wait_group_read_all();
      }
      __syncwarp();
#pragma unroll
      for (uint32_t j = 0; j < 8; ++j)
        sts_u4(row_addr + ((j ^ sw) << 4), a1[4 * j], a1[4 * j + 1], a1[4 * j + 2], a1[4 * j + 3]);
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0 && row0 < p.Tq) {
        tma_reduce_add_4d(box, &tm_dqacc, 32, row0, h, b);
        bulk_commit_group();
      }
    }
    if (lane == 0) bulk_wait_group_all();
  } else {
    // Elementwise warps: thread = key row of the tile = TMEM lane; this warp covers query
    // columns [64 * half, 64 * half + 64) of each step, as two chunks of 32.
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const int key = k0 + r;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_base + T_ST + half * 64;
    const uint32_t t_dp = tmem + lane_base + T_DPT + half * 64;
    const uint32_t t_p = tmem + lane_base + T_P + half * 32;
    const uint32_t ds_row = smem_u32(s.ds[half]) + r * 128;
    const uint32_t sw = static_cast<uint32_t>(r & 7);
    bool ok = true;
    for (int i = 0; i < n_q; ++i) {
      const int st = i % STAGES;
      const long long q0 = static_cast<long long>(qt0 + i) * T;
      const uint32_t nl_addr = smem_u32(&s.nlse2[st][half * 64]);
      const uint32_t nd_addr = smem_u32(&s.nd[st][half * 64]);
      // Pair (key, q) is visible iff q >= key - past_len; only steps crossing the diagonal mask.
      const bool masked = static_cast<long long>(k0) + T - 1 > q0 + p.past_len;
      const int first_visible = static_cast<int>(min(static_cast<long long>(T),
          max(0LL, key - p.past_len - q0))) - half * 64;  // column of this warp's 64

      // Phase 1: P from S^T.
      if (!warp_wait(s, &s.s_full, i & 1)) { ok = false; break; }
      tc_fence_after();
      float pr[64];
      {
        uint32_t sr0[32], sr1[32];
        tmem_ld32(t_s, sr0);
        tmem_ld32(t_s + 32, sr1);
        tmem_wait_ld();
        reg_fence(sr0);
        reg_fence(sr1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.s_consumed);
        // P^T(i - 1) has been read by dV(i - 1) (long done by now, normally).
        if (i > 0 && !warp_wait(s, &s.pv_free, (i - 1) & 1)) { ok = false; break; }
        tc_fence_after();
        uint32_t pk[16];
        if (masked) ew_probs<true>(sr0, nl_addr, first_visible, pr, pk);
        else ew_probs<false>(sr0, nl_addr, 0, pr, pk);
        tmem_st16(t_p, pk);
        if (masked) ew_probs<true>(sr1, nl_addr + 128, first_visible - 32, pr + 32, pk);
        else ew_probs<false>(sr1, nl_addr + 128, 0, pr + 32, pk);
        tmem_st16(t_p + 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.p_full);

      // Phase 2: dS from dP^T and the FP32 P, 16 queries at a time.
      if (!warp_wait(s, &s.dp_full, i & 1)) { ok = false; break; }
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t dr[16], dsb[8];
        tmem_ld16(t_dp + 16 * c, dr);
        tmem_wait_ld();
        reg_fence16(dr);
        ew_dscores(pr + 16 * c, dr, nd_addr + 64 * c, dsb);
        // The dS tile was last read by dQ(i - 1).
        if (c == 0 && i > 0 && !warp_wait(s, &s.ds_free, (i - 1) & 1)) {
          ok = false;
          break;
        }
        const uint32_t j = 2 * c;  // 8-query chunks j, j + 1 of the half
        sts_u4(ds_row + ((j ^ sw) << 4), dsb[0], dsb[1], dsb[2], dsb[3]);
        sts_u4(ds_row + (((j + 1) ^ sw) << 4), dsb[4], dsb[5], dsb[6], dsb[7]);
      }
      if (!ok) break;
      fence_proxy_async_smem();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.ds_ready);
    }
    if (ok && warp_wait(s, &s.acc_final, 0)) {
      tc_fence_after();
      // Warps 0-3 write dK, warps 4-7 dV (same TMEM lanes, different columns).
      const size_t kidx = static_cast<size_t>(bh) * p.Tk + static_cast<size_t>(key);
      const uint32_t col = half == 0 ? T_DK : T_DV;
      __nv_bfloat16* out = half == 0 ? p.dk : p.dv;
      const float scale = half == 0 ? SCALE : 1.f;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t acc[32];
        tmem_ld32(tmem + lane_base + col + c * 32, acc);
        tmem_wait_ld();
        reg_fence(acc);
        if (key < p.Tk) store_row_bf16(out + kidx * HD + c * 32, acc, scale);
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

// dQ = bf16(scale * dQ_acc), eight features per thread.
struct ConvertParams {
  long long rows;       // B * H * Tq
  const float* acc;     // [rows, 64]
  __nv_bfloat16* dq;    // [rows, 64]
};

__global__ void __launch_bounds__(256) bwd_dq_convert_kernel(const ConvertParams p) {
  const long long i = static_cast<long long>(blockIdx.x) * 256 + threadIdx.x;  // 8-feature group
  if (i >= p.rows * (HD / 8)) return;
  const float4 a = reinterpret_cast<const float4*>(p.acc)[2 * i];
  const float4 c = reinterpret_cast<const float4*>(p.acc)[2 * i + 1];
  reinterpret_cast<uint4*>(p.dq)[i] =
      make_uint4(pack_bf16x2(a.x * SCALE, a.y * SCALE), pack_bf16x2(a.z * SCALE, a.w * SCALE),
                 pack_bf16x2(c.x * SCALE, c.y * SCALE), pack_bf16x2(c.z * SCALE, c.w * SCALE));
}

}  // namespace fused

// ------------------------------------------------------------------ persistent dQ/dK/dV kernel
// The fused kernel above as a persistent grid: one CTA per SM takes (b, h, 128-key tile) work
// items from a global counter (heaviest key tiles first, zeroed by bwd_preprocess_kernel) and
// runs them back to back. Per item the products, the elementwise phases and the dQ reduce are
// those of bwd_fused_kernel; what changes is what happens between items:
// * K and V sit in two slots: the TMA warp loads the next item's tiles while the current item
//   still runs (a slot is refilled once the last dQ product of its previous item has completed
//   and every role has read that item's index).
// * The Q / dO ring, S^T, dP^T, P^T, dS and the dQ step keep one step counter across items, so
//   the first scores of the next item are computed under the last steps of the current one.
// * The four drain warps write dK and dV (after the item's last dQ step) instead of the
//   elementwise warps, which go straight on to the next item; the first dV / dK product of the
//   next item waits for that read (acc_empty).
// Every wait is bounded, as in the other kernels.
namespace persist {

using fused::DQ_BOX_ROWS;
using fused::DQ_WARP0;
using fused::EW_WARPS;
using fused::LOAD_WARP;
using fused::MMA_WARP;
using fused::SCORE_WARP;
using fused::STAGES;
using fused::T;
using fused::T_DK;
using fused::T_DPT;
using fused::T_DQ;
using fused::T_DV;
using fused::T_P;
using fused::T_ST;
using fused::THREADS;
using fused::TILE_BYTES;
using fused::TMEM_COLS;

constexpr int KV_SLOTS = 2;

struct Params {
  int B, H, Tq, Tk, past_len;
  int n_k_tiles;
  int Tq_pad;               // Tq rounded up to whole 128-row tiles
  int n_items;              // B * H * n_k_tiles
  const float* nlse2;       // [B, H, Tq_pad]: -LSE * log2(e), -inf on padding rows
  const float* nd;          // [B, H, Tq_pad]: -D
  __nv_bfloat16* dk;        // contiguous [B, H, Tk, 64]
  __nv_bfloat16* dv;
  unsigned int* next_item;  // work counter, zero at launch
};

struct alignas(1024) Smem {
  uint8_t k[KV_SLOTS][TILE_BYTES];
  uint8_t v[KV_SLOTS][TILE_BYTES];
  uint8_t q[STAGES][TILE_BYTES];
  uint8_t dO[STAGES][TILE_BYTES];
  uint8_t ds[2][T * 128];  // as in bwd_fused_kernel
  uint8_t dq_stage[4][DQ_BOX_ROWS * 128];
  float nlse2[STAGES][T];
  float nd[STAGES][T];
  volatile int item[KV_SLOTS];  // work item of the slot, -1 once the counter ran out
  uint64_t kv_full[KV_SLOTS], kv_empty[KV_SLOTS];
  uint64_t q_full[STAGES], q_empty[STAGES];
  uint64_t s_full, s_consumed, p_full, pv_free, dp_full, ds_ready, ds_free;
  uint64_t dq_full, dq_free, acc_final, acc_empty, drain, drain_scores;
  uint32_t tmem_base;
  volatile int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 1024;
static_assert(kSmemBytes <= 227 * 1024, "persistent backward shared memory");

// kv_empty of a slot: the commit after the item's last dQ product plus one arrival per drain
// warp once it has read the item's index (the drain warps are the only role that can still be
// an item behind when the slot is refilled).
constexpr int KV_EMPTY_ARRIVALS = 1 + 4;

struct Item {
  int bh, b, h, k0, qt0, n_q;
};

__device__ __forceinline__ Item decode_item(const Params& p, int idx) {
  const int BH = p.B * p.H;
  Item it;
  const int kt = idx / BH;  // low key tiles see the most queries: heaviest first
  it.bh = idx - kt * BH;
  it.b = it.bh / p.H;
  it.h = it.bh - it.b * p.H;
  it.k0 = kt * T;
  it.qt0 = static_cast<int>(max(0LL, static_cast<long long>(it.k0) - p.past_len) / T);
  it.n_q = (p.Tq + T - 1) / T - it.qt0;
  return it;
}

__global__ void __launch_bounds__(THREADS, 1)
bwd_persistent_kernel(const __grid_constant__ CUtensorMap tm_q,
                      const __grid_constant__ CUtensorMap tm_k,
                      const __grid_constant__ CUtensorMap tm_v,
                      const __grid_constant__ CUtensorMap tm_do,
                      const __grid_constant__ CUtensorMap tm_dqacc, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < KV_SLOTS; ++i) {
      mbar_init(&s.kv_full[i], 1);
      mbar_init(&s.kv_empty[i], KV_EMPTY_ARRIVALS);
    }
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.q_full[i], 1);
      mbar_init(&s.q_empty[i], 1);
    }
    mbar_init(&s.s_full, 1);
    mbar_init(&s.s_consumed, EW_WARPS);
    mbar_init(&s.p_full, EW_WARPS);
    mbar_init(&s.pv_free, 1);
    mbar_init(&s.dp_full, 1);
    mbar_init(&s.ds_ready, EW_WARPS);
    mbar_init(&s.ds_free, 1);
    mbar_init(&s.dq_full, 1);
    mbar_init(&s.dq_free, 4);
    mbar_init(&s.acc_final, 1);
    mbar_init(&s.acc_empty, 4);
    mbar_init(&s.drain, 1);
    mbar_init(&s.drain_scores, 1);
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
      int items = 0;  // items whose K/V loads were issued
      int g = 0;      // Q / dO ring loads issued
      bool ok = true;
      for (int j = 0; ok; ++j) {
        const int slot = j & 1;
        if (j >= KV_SLOTS && !wait_or_abort(s, &s.kv_empty[slot], ((j >> 1) - 1) & 1)) break;
        // Compared unsigned: the counter passes n_items by up to one grab per CTA.
        const unsigned int grab = atomicAdd(p.next_item, 1u);
        if (grab >= static_cast<unsigned int>(p.n_items)) {
          s.item[slot] = -1;
          mbar_arrive(&s.kv_full[slot]);
          break;
        }
        const int idx = static_cast<int>(grab);
        s.item[slot] = idx;
        const Item it = decode_item(p, idx);
        mbar_arrive_expect_tx(&s.kv_full[slot], 2 * TILE_BYTES);
        tma_load_4d(s.k[slot], &tm_k, &s.kv_full[slot], 0, it.k0, it.h, it.b);
        tma_load_4d(s.v[slot], &tm_v, &s.kv_full[slot], 0, it.k0, it.h, it.b);
        items = j + 1;
        for (int i = 0; i < it.n_q; ++i) {
          const int st = g % STAGES;
          if (g >= STAGES && !wait_or_abort(s, &s.q_empty[st], ((g / STAGES) - 1) & 1)) {
            ok = false;
            break;
          }
          const int q0 = (it.qt0 + i) * T;
          const size_t row = static_cast<size_t>(it.bh) * p.Tq_pad + static_cast<size_t>(q0);
          mbar_arrive_expect_tx(&s.q_full[st], 2 * TILE_BYTES + 2 * T * sizeof(float));
          tma_load_4d(s.q[st], &tm_q, &s.q_full[st], 0, q0, it.h, it.b);
          tma_load_4d(s.dO[st], &tm_do, &s.q_full[st], 0, q0, it.h, it.b);
          bulk_load_plain(s.nlse2[st], p.nlse2 + row, T * sizeof(float), &s.q_full[st]);
          bulk_load_plain(s.nd[st], p.nd + row, T * sizeof(float), &s.q_full[st]);
          ++g;
        }
      }
      if (s.abort) {
        // Let the copies in flight land before the CTA's shared memory is released.
        for (int j = max(0, items - KV_SLOTS); j < items; ++j)
          mbar_wait(&s.kv_full[j & 1], (j >> 1) & 1);
        for (int i = max(0, g - STAGES); i < g; ++i)
          mbar_wait(&s.q_full[i % STAGES], (i / STAGES) & 1);
      }
    }
  } else if (warp == SCORE_WARP) {
    if (lane == 0) {
      const uint32_t idesc_s = make_idesc_bf16(T, T, false);
      bool ok = true;
      int g = 0;
      for (int j = 0; ok; ++j) {
        const int slot = j & 1;
        if (!wait_or_abort(s, &s.kv_full[slot], (j >> 1) & 1)) break;
        const int idx = s.item[slot];
        if (idx < 0) break;
        const Item it = decode_item(p, idx);
        const uint32_t k_addr = smem_u32(s.k[slot]), v_addr = smem_u32(s.v[slot]);
        for (int i = 0; i < it.n_q; ++i, ++g) {
          const int st = g % STAGES;
          // S^T(g) once the Q tile has landed and the elementwise warps hold S^T(g-1).
          ok = wait_or_abort(s, &s.q_full[st], (g / STAGES) & 1) &&
               (g == 0 || wait_or_abort(s, &s.s_consumed, (g - 1) & 1));
          if (!ok) break;
          tc_fence_after();
          issue_scores(tmem + T_ST, k_addr, smem_u32(s.q[st]), idesc_s);
          umma_commit(&s.s_full);
          // dP^T(g) overwrites dP^T(g-1): once the elementwise warps have read it.
          if (g > 0 && !wait_or_abort(s, &s.ds_ready, (g - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_scores(tmem + T_DPT, v_addr, smem_u32(s.dO[st]), idesc_s);
          umma_commit(&s.dp_full);
        }
      }
      umma_commit(&s.drain_scores);
      mbar_wait(&s.drain_scores, 0);
    }
  } else if (warp == MMA_WARP) {
    if (lane == 0) {
      const uint32_t idesc_o = make_idesc_bf16(T, HD, true);
      const uint32_t idesc_dq = make_idesc_bf16(T, HD, true) | (1u << 15);  // A MN-major
      bool ok = true;
      int g = 0;
      for (int j = 0; ok; ++j) {
        const int slot = j & 1;
        if (!wait_or_abort(s, &s.kv_full[slot], (j >> 1) & 1)) break;
        const int idx = s.item[slot];
        if (idx < 0) break;
        const Item it = decode_item(p, idx);
        const uint32_t k_addr = smem_u32(s.k[slot]);
        for (int i = 0; i < it.n_q; ++i, ++g) {
          const int st = g % STAGES;
          ok = wait_or_abort(s, &s.p_full, g & 1) &&
               // The first products of an item overwrite dV and dK: after the drain warps
               // have read the previous item's.
               (i > 0 || j == 0 || wait_or_abort(s, &s.acc_empty, (j - 1) & 1));
          if (!ok) break;
          tc_fence_after();
          fused::issue_dv(tmem + T_DV, tmem + T_P, smem_u32(s.dO[st]), idesc_o, i > 0);
          umma_commit(&s.pv_free);
          if (!wait_or_abort(s, &s.ds_ready, g & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fused::issue_dk(tmem + T_DK, smem_u32(s.ds[0]), smem_u32(s.q[st]), idesc_o, i > 0);
          // Q(g) and dO(g) were last read by dK(g) and dV(g); S^T(g) and dP^T(g) completed
          // before the elementwise warps could read them.
          umma_commit(&s.q_empty[st]);
          if (i + 1 == it.n_q) umma_commit(&s.acc_final);
          if (g > 0 && !wait_or_abort(s, &s.dq_free, (g - 1) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          fused::issue_dq(tmem + T_DQ, smem_u32(s.ds[0]), k_addr, idesc_dq);
          umma_commit(&s.dq_full);
          umma_commit(&s.ds_free);
          // K was last read by this dQ product, V by dP^T (complete before dS existed).
          if (i + 1 == it.n_q) umma_commit(&s.kv_empty[slot]);
        }
      }
      umma_commit(&s.drain);
      mbar_wait(&s.drain, 0);
    }
  } else if (warp >= DQ_WARP0 && warp < DQ_WARP0 + 4) {
    // dQ drain for every step (thread = query row 32 * quarter + lane of the step), then the
    // item's dK and dV rows (thread = key row 32 * quarter + lane; same TMEM lanes).
    const int quarter = warp & 3;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    uint8_t* box = s.dq_stage[quarter];
    const uint32_t sw = lane & 7;
    const uint32_t row_addr = smem_u32(box) + lane * 128;
    bool ok = true;
    int g = 0;
    for (int j = 0; ok; ++j) {
      const int slot = j & 1;
      if (!warp_wait(s, &s.kv_full[slot], (j >> 1) & 1)) break;
      const int idx = s.item[slot];
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.kv_empty[slot]);
      if (idx < 0) break;
      const Item it = decode_item(p, idx);
      for (int i = 0; i < it.n_q; ++i, ++g) {
        if (!warp_wait(s, &s.dq_full, g & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t a0[32], a1[32];
        tmem_ld32(tmem + lane_base + T_DQ, a0);
        tmem_ld32(tmem + lane_base + T_DQ + 32, a1);
        tmem_wait_ld();
        reg_fence(a0);
        reg_fence(a1);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&s.dq_free);
          bulk_wait_group_read_all();  // the previous reduce has read the staging box
        }
        __syncwarp();
        const int row0 = (it.qt0 + i) * T + quarter * DQ_BOX_ROWS;
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c)
          sts_u4(row_addr + ((c ^ sw) << 4), a0[4 * c], a0[4 * c + 1], a0[4 * c + 2], a0[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < p.Tq) {  // rows past Tq inside a box are clipped by the map
          tma_reduce_add_4d(box, &tm_dqacc, 0, row0, it.h, it.b);
          bulk_commit_group();
          bulk_wait_group_read_all();
        }
        __syncwarp();
#pragma unroll
        for (uint32_t c = 0; c < 8; ++c)
          sts_u4(row_addr + ((c ^ sw) << 4), a1[4 * c], a1[4 * c + 1], a1[4 * c + 2], a1[4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0 && row0 < p.Tq) {
          tma_reduce_add_4d(box, &tm_dqacc, 32, row0, it.h, it.b);
          bulk_commit_group();
        }
      }
      if (!ok || !warp_wait(s, &s.acc_final, j & 1)) break;
      tc_fence_after();
      const int key = it.k0 + quarter * 32 + lane;
      const size_t kidx = static_cast<size_t>(it.bh) * p.Tk + static_cast<size_t>(key);
#pragma unroll
      for (int part = 0; part < 2; ++part) {  // dK (scaled), then dV
        uint32_t a0[32], a1[32];
        tmem_ld32(tmem + lane_base + (part == 0 ? T_DK : T_DV), a0);
        tmem_ld32(tmem + lane_base + (part == 0 ? T_DK : T_DV) + 32, a1);
        tmem_wait_ld();
        reg_fence(a0);
        reg_fence(a1);
        if (part == 1) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.acc_empty);
        }
        __nv_bfloat16* out = part == 0 ? p.dk : p.dv;
        const float scale = part == 0 ? SCALE : 1.f;
        if (key < p.Tk) {
          store_row_bf16(out + kidx * HD, a0, scale);
          store_row_bf16(out + kidx * HD + 32, a1, scale);
        }
      }
    }
    if (lane == 0) bulk_wait_group_all();
  } else {
    // Elementwise warps: thread = key row of the item's tile = TMEM lane; this warp covers
    // query columns [64 * half, 64 * half + 64) of each step, as in bwd_fused_kernel.
    const int quarter = warp & 3, half = warp >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t t_s = tmem + lane_base + T_ST + half * 64;
    const uint32_t t_dp = tmem + lane_base + T_DPT + half * 64;
    const uint32_t t_p = tmem + lane_base + T_P + half * 32;
    const uint32_t ds_row = smem_u32(s.ds[half]) + r * 128;
    const uint32_t sw = static_cast<uint32_t>(r & 7);
    bool ok = true;
    int g = 0;
    for (int j = 0; ok; ++j) {
      const int slot = j & 1;
      if (!warp_wait(s, &s.kv_full[slot], (j >> 1) & 1)) break;
      const int idx = s.item[slot];
      if (idx < 0) break;
      const Item it = decode_item(p, idx);
      const int key = it.k0 + r;
      for (int i = 0; i < it.n_q; ++i, ++g) {
        const int st = g % STAGES;
        const long long q0 = static_cast<long long>(it.qt0 + i) * T;
        const uint32_t nl_addr = smem_u32(&s.nlse2[st][half * 64]);
        const uint32_t nd_addr = smem_u32(&s.nd[st][half * 64]);
        const bool masked = static_cast<long long>(it.k0) + T - 1 > q0 + p.past_len;
        const int first_visible = static_cast<int>(min(static_cast<long long>(T),
            max(0LL, key - p.past_len - q0))) - half * 64;

        // Phase 1: P from S^T.
        if (!warp_wait(s, &s.s_full, g & 1)) { ok = false; break; }
        tc_fence_after();
        float pr[64];
        {
          uint32_t sr0[32], sr1[32];
          tmem_ld32(t_s, sr0);
          tmem_ld32(t_s + 32, sr1);
          tmem_wait_ld();
          reg_fence(sr0);
          reg_fence(sr1);
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&s.s_consumed);
          // P^T(g - 1) has been read by dV(g - 1).
          if (g > 0 && !warp_wait(s, &s.pv_free, (g - 1) & 1)) { ok = false; break; }
          tc_fence_after();
          uint32_t pk[16];
          if (masked) fused::ew_probs<true>(sr0, nl_addr, first_visible, pr, pk);
          else fused::ew_probs<false>(sr0, nl_addr, 0, pr, pk);
          tmem_st16(t_p, pk);
          if (masked) fused::ew_probs<true>(sr1, nl_addr + 128, first_visible - 32, pr + 32, pk);
          else fused::ew_probs<false>(sr1, nl_addr + 128, 0, pr + 32, pk);
          tmem_st16(t_p + 16, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.p_full);

        // Phase 2: dS from dP^T and the FP32 P, 16 queries at a time.
        if (!warp_wait(s, &s.dp_full, g & 1)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t dr[16], dsb[8];
          tmem_ld16(t_dp + 16 * c, dr);
          tmem_wait_ld();
          reg_fence16(dr);
          fused::ew_dscores(pr + 16 * c, dr, nd_addr + 64 * c, dsb);
          // The dS tile was last read by dK(g - 1) and dQ(g - 1).
          if (c == 0 && g > 0 && !warp_wait(s, &s.ds_free, (g - 1) & 1)) {
            ok = false;
            break;
          }
          const uint32_t q8 = 2 * c;  // 8-query chunks q8, q8 + 1 of the half
          sts_u4(ds_row + ((q8 ^ sw) << 4), dsb[0], dsb[1], dsb[2], dsb[3]);
          sts_u4(ds_row + (((q8 + 1) ^ sw) << 4), dsb[4], dsb[5], dsb[6], dsb[7]);
        }
        if (!ok) break;
        fence_proxy_async_smem();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.ds_ready);
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

}  // namespace persist

}  // namespace backward
}  // namespace tt
