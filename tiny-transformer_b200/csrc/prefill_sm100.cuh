// BF16 causal attention forward (prefill / chunked prefill) for sm_100a.
//
// Semantics follow the reference operator (tiny_transformer/operators/reference.py:37-53 and
// csrc/attention/attention_forward_BF16_kernel.cuh:232-389 in Tiny-transformer):
//   key j is visible to query row i iff j <= i + past_len (inclusive causal, Tk == past_len + Tq),
//   softmax scale 1/sqrt(64), FP32 softmax, P rounded to BF16 before P.V,
//   O in BF16, LSE = natural-log logsumexp of the scaled scores in FP32.
//
// One CTA (one per SM) computes a 256-row query block of one (batch, head) as two 128-row
// tiles t = 0, 1 that share every K/V tile the producer loads. Roles (3 warpgroups):
//   warps 0-3   softmax + epilogue of tile 0 (thread = query row = TMEM lane)
//   warps 4-7   softmax + epilogue of tile 1
//   warp  8     TMA producer: Q tiles once, then K/V tiles through a STAGES-deep ring
//   warp  9     S issuer for both tiles: S_t(j) = Q_t.K(j)^T into the next free score buffer
//   warps 10,11 P.V issuers, one per query tile t: O_t += P_t(j).V(j) (P from TMEM) once the
//               softmax publishes P_t(j). A tcgen05.mma blocks its issuing thread while the
//               tensor core's queue is full (~100 cycles per instruction under load), so the S
//               stream must not queue behind a P.V issue: separate threads keep the next S
//               from waiting on the previous tile's P.V.
// Score buffers: the (KV tile j, query tile t) pairs are numbered in issue order ("slots":
// per KV tile, tile 1 then tile 0) and slot s uses TMEM buffer s % 3. The softmax writes
// P (bf16x2) over the first 64 columns of its own scores, so it never waits for the previous
// P.V before publishing P, and the S of slot s + 3 is issued once the P.V of slot s has read
// its buffer: the tensor core computes the next scores of a tile while its softmax still works
// on the current ones, and one slow warp no longer holds back the next S of its tile.
// Registers: launched at 168 per thread (384 threads, the 64K register file); the producer
// warpgroup drops to 88 and the softmax warpgroups rise to 208 (2 x 208 + 88 = 504 <= 3 x 168;
// with P stored in 32-score chunks the softmax needs no more, and the issuers' slot
// bookkeeping spills below 88).
// TMEM (all 512 columns): score / P buffers at [128b, 128b + 128) for b = 0, 1, 2, O_t at
// 384 + 64t.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cstdint>
#include <type_traits>

#include "sm100_ptx.cuh"

namespace tt {
namespace prefill {

constexpr int BM = 128;                 // query rows per tile (UMMA M)
constexpr int TILES = 2;                // query tiles per CTA
constexpr int BLOCK_M = BM * TILES;     // query rows per CTA
constexpr int BN = 128;                 // keys per KV tile (UMMA N of S)
constexpr int HD = 64;                  // head dim
constexpr int STAGES = 3;               // K/V ring depth
constexpr int SOFTMAX_WARPS = 4 * TILES;
constexpr int LOAD_WARP = SOFTMAX_WARPS;
constexpr int MMA_WARP = SOFTMAX_WARPS + 1;  // S issuer; MMA_WARP + 1 + t issues P.V of tile t
constexpr int THREADS = (SOFTMAX_WARPS + 4) * 32;  // three full warpgroups
constexpr uint32_t LAUNCH_REGS = 168;    // registers per thread at launch (65536 / 384, rounded)
constexpr uint32_t SOFTMAX_REGS = 208;
constexpr uint32_t PRODUCER_REGS = 88;
static_assert(2 * SOFTMAX_REGS + PRODUCER_REGS <= 3 * LAUNCH_REGS,
              "register hand-over exceeds the launch allocation");
static_assert(THREADS * LAUNCH_REGS <= 65536, "launch allocation exceeds the register file");
constexpr uint32_t TILE_BYTES = BM * HD * 2;  // 16 KiB, one 128x64 bf16 tile
constexpr uint32_t TMEM_COLS = 512;
constexpr int SBUF = 3;                  // rotating score / P buffers shared by both tiles
constexpr uint32_t O_COL = SBUF * BN;    // O_t at O_COL + 64t
static_assert(O_COL + TILES * HD <= TMEM_COLS, "TMEM layout exceeds 512 columns");
constexpr float LN2 = 0.69314718055994530942f;
// O is rescaled only when the running row max grows by more than this (log2 units);
// between rescales P stays below 2^8, far inside the FP32/BF16 range.
constexpr float RESCALE_THRESHOLD = 8.0f;

struct alignas(1024) Smem {
  uint8_t q[TILES][TILE_BYTES];
  uint8_t k[STAGES][TILE_BYTES];
  uint8_t v[STAGES][TILE_BYTES];
  uint64_t q_full;
  uint64_t k_full[STAGES], k_empty[STAGES];
  uint64_t v_full[STAGES], v_empty[STAGES];
  uint64_t s_full[SBUF];   // scores of the buffer's current slot are in TMEM
  uint64_t p_ready[SBUF];  // its P is in TMEM (and O rescaled if needed): 4 warp arrivals
  uint64_t buf_free[SBUF]; // the P.V that read the buffer's P has completed
  uint64_t o_done[TILES];  // P.V of tile t completed (once per KV tile)
  uint64_t drain[TILES + 1];  // one per issuing thread
  uint32_t tmem_base;
  volatile int abort;
};

constexpr size_t kSmemBytes = sizeof(Smem) + 1024;  // + slack for 1 KiB alignment

// Record of one query row's partial result over one part of its KV range (split query
// blocks only): unnormalised O[64], running max m (log2 units), row sum l, 2 pad (16-byte
// aligned records).
constexpr int PART_REC = HD + 4;

struct Params {
  int B, H, Tq, Tk, past_len;
  int n_qblocks;     // ceil(Tq / BLOCK_M)
  __nv_bfloat16* o;  // contiguous [B, H, Tq, 64]
  float* lse;        // contiguous [B, H, Tq]
  float scale_log2;  // softmax scale * log2(e)
  // KV split of query blocks (few CTAs for the SMs): a block of n KV tiles runs as
  // parts = ceil(n / part_tiles) CTAs over consecutive, near-equal KV ranges
  // [i * n / parts, (i + 1) * n / parts), each writing partial records that
  // prefill_combine_kernel merges. part_tiles = 0: no split.
  int part_tiles;
  int max_parts;          // parts of the longest block (record stride), at most 32
  int first_split_qb;     // lowest query block that is split
  float* partials;        // [B*H, n_qblocks, max_parts, BLOCK_M, PART_REC]
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

// Number of KV tiles query rows [q0, q0 + BM) need: keys up to q0 + BM - 1 + past_len.
__device__ __forceinline__ int kv_tiles_for(const Params& p, int q0) {
  if (q0 >= p.Tq) return 0;
  const long long end =
      min(static_cast<long long>(p.Tk), static_cast<long long>(q0) + BM + p.past_len);
  return static_cast<int>((end + BN - 1) / BN);
}

// KV tiles query block qb loads (its second tile needs at least as many as its first unless
// it lies past Tq).
__device__ __forceinline__ int block_tiles(const Params& p, int qb) {
  return max(kv_tiles_for(p, qb * BLOCK_M), kv_tiles_for(p, qb * BLOCK_M + BM));
}

__device__ __forceinline__ int block_parts(const Params& p, int qb) {
  return p.part_tiles == 0 ? 1 : max(1, (block_tiles(p, qb) + p.part_tiles - 1) / p.part_tiles);
}

__device__ __forceinline__ float* part_record(const Params& p, int bh, int qb, int part,
                                              int row_in_block) {
  return p.partials +
         ((static_cast<size_t>(bh) * p.n_qblocks + qb) * p.max_parts + part) * BLOCK_M * PART_REC +
         static_cast<size_t>(row_in_block) * PART_REC;
}

// Issue-order number of the pair (KV tile j, query tile t): per KV tile, tile 1 (if it needs
// j) then tile 0 (if it needs j). Tile 1 needs at least as many KV tiles as tile 0 unless it
// lies past Tq (n1 == 0), so the pairs before (j, t) are min(j, n0) + min(j, n1), plus tile 1's
// pair of the same KV tile when t == 0.
__device__ __forceinline__ int slot_of(int j, int t, int n0, int n1) {
  return min(j, n0) + min(j, n1) + ((t == 0 && j < n1) ? 1 : 0);
}

// Row maximum of the 128 scores: a 3-input max tree, depth ~6 instead of a 127-long chain.
__device__ __forceinline__ float row_max(const float (&x)[BN]) {
  float a[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = fmax3(x[i], x[i + 16], x[i + 32]);
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = fmax3(a[i], x[i + 48], x[i + 64]);
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = fmax3(a[i], x[i + 80], x[i + 96]);
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = fmaxf(a[i], x[i + 112]);
  float b[6];
#pragma unroll
  for (int i = 0; i < 5; ++i) b[i] = fmax3(a[3 * i], a[3 * i + 1], a[3 * i + 2]);
  b[5] = a[15];
  return fmaxf(fmax3(b[0], b[1], b[2]), fmax3(b[3], b[4], b[5]));
}

// exp2 of two arguments on the FMA pipe, to take load off the MUFU unit (16 ex2 per clock
// per SM, the binding limit of a D = 64 softmax). Cody-Waite range reduction
// 2^x = 2^n * 2^f, n = round(x) by adding 1.5 * 2^23, f = x - n in [-1/2, 1/2]; 2^f by a
// degree-3 minimax polynomial with p(0) = 1 (coefficients from fit_exp2_poly.py; maximum
// relative error 1.02e-4 in FP32); n is added to the exponent field. Arguments are clamped
// at -127, which yields exactly +0.0, so masked (-inf) scores give exact zeros.
constexpr float kPolyC1 = 0.6932827f;    // 0x3f317afa
constexpr float kPolyC2 = 0.24221104f;   // 0x3e78062c
constexpr float kPolyC3 = 0.055009704f;  // 0x3d6151db
constexpr float kRoundMagic = 12582912.0f;  // 1.5 * 2^23

__device__ __forceinline__ void exp2_poly2(float a, float b, float& pa, float& pb) {
  const uint64_t x2 = f2_pack(fmaxf(a, -127.f), fmaxf(b, -127.f));
  const uint64_t t2 = f2_add(x2, f2_pack(kRoundMagic, kRoundMagic));
  const uint64_t r2 = f2_add(t2, f2_pack(-kRoundMagic, -kRoundMagic));
  const uint64_t f2 = f2_fma(r2, f2_pack(-1.f, -1.f), x2);
  uint64_t p2 = f2_fma(f2_pack(kPolyC3, kPolyC3), f2, f2_pack(kPolyC2, kPolyC2));
  p2 = f2_fma(p2, f2, f2_pack(kPolyC1, kPolyC1));
  p2 = f2_fma(p2, f2, f2_pack(1.f, 1.f));
  float q0, q1, n0, n1;
  f2_unpack(p2, q0, q1);
  f2_unpack(t2, n0, n1);
  pa = __uint_as_float(__float_as_uint(q0) + (__float_as_uint(n0) << 23));
  pb = __uint_as_float(__float_as_uint(q1) + (__float_as_uint(n1) << 23));
}

// Of every 8 consecutive score pairs, this many take the FMA-pipe exp2; the rest use MUFU.
constexpr int POLY_PAIRS_PER_8 = 3;

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

// p = exp2(x * sl2 - m) for the 128 scores of this row: packed f32x2 FMA for the argument,
// MUFU ex2 (or the FMA-pipe polynomial for POLY_PAIRS_PER_8 of every 8 pairs), bf16x2 packing,
// and the FP32 row sum over 8 independent packed accumulators. P goes to TMEM (16 columns per
// chunk of 32 scores) as soon as each chunk is packed, over the first 64 columns of the row's
// own score buffer (already read into x); the caller issues tcgen05.wait::st before publishing
// P. Returns the row sum.
__device__ __forceinline__ float exp_store_sum(const float (&x)[BN], float sl2, float m,
                                               uint32_t t_p) {
  const uint64_t sc2 = f2_pack(sl2, sl2);
  const uint64_t nm2 = f2_pack(-m, -m);
  uint64_t acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0;
#pragma unroll
  for (int chunk = 0; chunk < BN / 32; ++chunk) {
    uint32_t pk[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int c = chunk * 16 + i;
      float t0, t1;
      f2_unpack(f2_fma(f2_pack(x[2 * c], x[2 * c + 1]), sc2, nm2), t0, t1);
      float p0, p1;
      if ((c & 7) < POLY_PAIRS_PER_8) {
        exp2_poly2(t0, t1, p0, p1);
      } else {
        p0 = ex2_approx(t0);
        p1 = ex2_approx(t1);
      }
      acc[c & 7] = f2_add(acc[c & 7], f2_pack(p0, p1));
      pk[i] = pack_bf16x2(p0, p1);
    }
    tmem_st16(t_p + chunk * 16, pk);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) acc[i] = f2_add(acc[i], acc[i + 4]);
  acc[0] = f2_add(acc[0], acc[2]);
  acc[1] = f2_add(acc[1], acc[3]);
  acc[0] = f2_add(acc[0], acc[1]);
  float lo, hi;
  f2_unpack(acc[0], lo, hi);
  return lo + hi;
}

// Softmax + epilogue for query tile t (128 rows); executed by the 4 warps of that tile.
// The CTA covers KV tiles [k0, k0 + its steps); n0 / n1: the steps query tiles 0 / 1 take in
// it (they fix the slot numbering). A CTA of a split block (parts > 1) writes its rows'
// partial records instead of O and LSE.
template <bool SPLIT>
__device__ __forceinline__ void softmax_tile(Smem& s, const Params& p, uint32_t tmem, int t,
                                             int wq, int lane, int bh, int qb, int q0, int n0,
                                             int n1, int k0, int part, int parts) {
  const int n_kv = t == 0 ? n0 : n1;
  const int r = wq * 32 + lane;  // query row within the tile == TMEM lane
  const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
  const uint32_t t_o = tmem + lane_base + O_COL + t * HD;
  const long long row_limit = static_cast<long long>(q0) + r + p.past_len;  // last visible key
  const long long tile_limit = static_cast<long long>(q0) + p.past_len;     // row 0's limit
  const float sl2 = p.scale_log2;
  float m_run = -INFINITY;  // running max of scaled scores, log2 units
  float l_run = 0.f;        // running sum of exp2(x - m_run)
  bool ok = true;

  // One KV step j of this tile; `masked` (std::true_type / std::false_type) selects the causal
  // mask at compile time. Returns false when a wait gave up (the CTA is aborting).
  auto step = [&](auto masked, int j) -> bool {
    // j: step within this CTA's KV range; k0 + j: the KV tile.
    const int slot = slot_of(j, t, n0, n1);
    const int buf = slot % SBUF;
    const uint32_t use = static_cast<uint32_t>(slot / SBUF);
    const uint32_t t_s = tmem + lane_base + buf * BN;
    if (!warp_wait(s, &s.s_full[buf], use & 1)) return false;
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

    const long long kv0 = static_cast<long long>(k0 + j) * BN;
    if constexpr (decltype(masked)::value) {
#pragma unroll
      for (int c = 0; c < BN; ++c)
        if (kv0 + c > row_limit) x[c] = -INFINITY;
    }
    const float mx = row_max(x);
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
    const float rowsum = exp_store_sum(x, sl2, m_use, t_s);
    l_run = l_run * factor + rowsum;

    if (j > 0 && __any_sync(0xffffffffu, need)) {
      // O_t holds the P.V sums up to KV tile j - 1 once that P.V has completed; it must be
      // rescaled to the new running max before P.V of tile j (issued after p_ready) adds to it.
      if (!warp_wait(s, &s.o_done[t], (j - 1) & 1)) return false;
      tc_fence_after();
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
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.p_ready[buf]);
    return true;
  };
  // Interior KV tiles (every key visible to every row of the tile) and the diagonal tiles
  // are separate compile-time instantiations of the step: only the latter carry the mask.
  const int n_full = static_cast<int>(min(static_cast<long long>(n_kv),
                                         max(0LL, (tile_limit + 1) / BN - k0)));
  int jj = 0;
  for (; jj < n_full; ++jj)
    if (!step(std::false_type{}, jj)) { ok = false; break; }
  if (ok)
    for (; jj < n_kv; ++jj)
      if (!step(std::true_type{}, jj)) { ok = false; break; }

  const int row = q0 + r;
  if (SPLIT && parts > 1) {
    // Partial record of this row over this part: O and l relative to the running max m.
    // Every lane takes part in the waits and TMEM loads (warp-collective); only the stores of
    // rows past Tq are skipped. ok and n_kv are warp-uniform.
    if (!ok) return;
    float4* dst = reinterpret_cast<float4*>(part_record(p, bh, qb, part, t * BM + r));
    const bool store = row < p.Tq;
    if (n_kv == 0) {
      // No KV tile of this part is visible to the tile: an empty record.
      if (store) {
#pragma unroll
        for (int i = 0; i < HD / 4; ++i) dst[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        dst[HD / 4] = make_float4(-INFINITY, 0.f, 0.f, 0.f);
      }
      return;
    }
    if (!warp_wait(s, &s.o_done[t], (n_kv - 1) & 1)) return;
    tc_fence_after();
    uint32_t o[HD / 32][32];
#pragma unroll
    for (int c = 0; c < HD / 32; ++c) tmem_ld32(t_o + c * 32, o[c]);
    tmem_wait_ld();
#pragma unroll
    for (int c = 0; c < HD / 32; ++c) reg_fence(o[c]);
    if (store) {
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          dst[c * 8 + i] =
              make_float4(__uint_as_float(o[c][4 * i]), __uint_as_float(o[c][4 * i + 1]),
                          __uint_as_float(o[c][4 * i + 2]), __uint_as_float(o[c][4 * i + 3]));
      }
      dst[HD / 4] = make_float4(m_run, l_run, 0.f, 0.f);
    }
    return;
  }
  if (ok && n_kv > 0 && warp_wait(s, &s.o_done[t], (n_kv - 1) & 1)) {
    tc_fence_after();
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

// SPLIT: the KV split of few, long query blocks (a separate instantiation, so the common
// unsplit kernel carries none of its bookkeeping).
template <bool SPLIT>
__global__ void __launch_bounds__(THREADS, 1)
attention_prefill_kernel(const __grid_constant__ CUtensorMap tm_q,
                         const __grid_constant__ CUtensorMap tm_k,
                         const __grid_constant__ CUtensorMap tm_v, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                     ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Heaviest causal blocks first: blocks are dispatched roughly in index order. With a KV
  // split, CTA i is part i / BH of the block's parts (per block, from the heaviest block down).
  const int BH = p.B * p.H;
  int qb, bh, part = 0, parts = 1;
  if (!SPLIT) {
    qb = p.n_qblocks - 1 - static_cast<int>(blockIdx.x / BH);
    bh = static_cast<int>(blockIdx.x % BH);
  } else {
    int idx = static_cast<int>(blockIdx.x);
    qb = p.n_qblocks - 1;
    for (; qb > 0; --qb) {
      const int np = block_parts(p, qb);
      if (idx < np * BH) break;
      idx -= np * BH;
    }
    parts = block_parts(p, qb);
    part = idx / BH;
    bh = idx - part * BH;
  }
  const int b = bh / p.H;
  const int h = bh % p.H;
  int q0[TILES], n_kv[TILES];
#pragma unroll
  for (int t = 0; t < TILES; ++t) {
    q0[t] = qb * BLOCK_M + t * BM;
    n_kv[t] = kv_tiles_for(p, q0[t]);
  }
  // Tile 1 never needs fewer KV tiles than tile 0 unless it lies past Tq (then it needs none).
  // This CTA's KV tiles [k0, k0 + n_load); per query tile, the steps it takes among them.
  int k0 = 0;
  int n_load = max(n_kv[0], n_kv[1]);
  if constexpr (SPLIT) {
    k0 = part * n_load / parts;
    n_load = (part + 1) * n_load / parts - k0;
#pragma unroll
    for (int t = 0; t < TILES; ++t) n_kv[t] = max(0, min(n_kv[t] - k0, n_load));
  }

  if (threadIdx.x == 0) {
    mbar_init(&s.q_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.k_full[i], 1);
      mbar_init(&s.k_empty[i], TILES);  // released by both tiles' issuers
      mbar_init(&s.v_full[i], 1);
      mbar_init(&s.v_empty[i], TILES);
    }
    for (int b = 0; b < SBUF; ++b) {
      mbar_init(&s.s_full[b], 1);
      mbar_init(&s.p_ready[b], 4);  // the 4 softmax warps of the slot's tile
      mbar_init(&s.buf_free[b], 1);
    }
    for (int t = 0; t < TILES; ++t) {
      mbar_init(&s.o_done[t], 1);
      mbar_init(&s.drain[t], 1);
    }
    mbar_init(&s.drain[TILES], 1);
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

  if (warp >= SOFTMAX_WARPS) {
    // Producer warpgroup: give registers to the softmax warpgroups, then split by warp.
    regs_decrease<PRODUCER_REGS>();
    if (warp == LOAD_WARP && lane == 0) {
      int issued_k = 0, issued_v = 0;  // K / V tiles whose loads were issued
      const int q_tiles = q0[1] < p.Tq ? 2 : 1;
      mbar_arrive_expect_tx(&s.q_full, q_tiles * TILE_BYTES);
      for (int t = 0; t < q_tiles; ++t) tma_load_4d(s.q[t], &tm_q, &s.q_full, 0, q0[t], h, b);
      for (int j = 0; j < n_load; ++j) {
        const int st = j % STAGES;
        const uint32_t use = j / STAGES;
        if (j >= STAGES && !wait_or_abort(s, &s.k_empty[st], (use - 1) & 1)) break;
        mbar_arrive_expect_tx(&s.k_full[st], TILE_BYTES);
        tma_load_4d(s.k[st], &tm_k, &s.k_full[st], 0, (k0 + j) * BN, h, b);
        issued_k = j + 1;
        if (j >= STAGES && !wait_or_abort(s, &s.v_empty[st], (use - 1) & 1)) break;
        mbar_arrive_expect_tx(&s.v_full[st], TILE_BYTES);
        tma_load_4d(s.v[st], &tm_v, &s.v_full[st], 0, (k0 + j) * BN, h, b);
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
    } else if (warp == MMA_WARP && lane == 0) {
      // S issuer for both query tiles, in slot order. A tile that does not need KV tile j (the
      // first one lies on the diagonal, the second past Tq) still releases the K stage once.
      // Tile 1 is served first: on diagonal blocks it has one more KV tile, so its chain ends
      // the CTA. The S of a slot goes into buffer slot % 3 once the P.V that read that
      // buffer's previous P (slot - 3) has completed.
      const uint32_t idesc_s = make_idesc_bf16(BM, BN, false);
      bool ok = wait_or_abort(s, &s.q_full, 0);
      for (int j = 0; ok && j < n_load; ++j) {
        const int st = j % STAGES;
        if (!wait_or_abort(s, &s.k_full[st], (j / STAGES) & 1)) break;
        for (int tt = 0; tt < TILES; ++tt) {
          const int t = TILES - 1 - tt;
          if (j < n_kv[t]) {
            const int slot = slot_of(j, t, n_kv[0], n_kv[1]);
            const int buf = slot % SBUF;
            const uint32_t use = static_cast<uint32_t>(slot / SBUF);
            if (use > 0 && !wait_or_abort(s, &s.buf_free[buf], (use - 1) & 1)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s_mma(tmem + buf * BN, smem_u32(s.q[t]), smem_u32(s.k[st]), idesc_s);
            umma_commit(&s.s_full[buf]);
            umma_commit(&s.k_empty[st]);
          } else {
            mbar_arrive(&s.k_empty[st]);
          }
        }
      }
      // All MMAs issued by this thread have completed once its drain barrier flips.
      umma_commit(&s.drain[TILES]);
      mbar_wait(&s.drain[TILES], 0);
    } else if (warp > MMA_WARP && warp <= MMA_WARP + TILES && lane == 0) {
      // P.V issuer of query tile t; afterwards it releases the V stages of KV tiles this tile
      // does not need (in order, each after it has been filled, so every stage counts exactly
      // one release per tile and use).
      const int t = warp - MMA_WARP - 1;
      const int n = n_kv[t];
      const uint32_t idesc_o = make_idesc_bf16(BM, HD, true);
      const uint32_t t_o = tmem + O_COL + t * HD;
      for (int j = 0; j < n; ++j) {
        const int st = j % STAGES;
        const int slot = slot_of(j, t, n_kv[0], n_kv[1]);
        const int buf = slot % SBUF;
        const uint32_t use = static_cast<uint32_t>(slot / SBUF);
        if (!wait_or_abort(s, &s.v_full[st], (j / STAGES) & 1)) break;
        if (!wait_or_abort(s, &s.p_ready[buf], use & 1)) break;
        tc_fence_after();
        issue_pv_mma(t_o, tmem + buf * BN, smem_u32(s.v[st]), idesc_o, j > 0);
        umma_commit(&s.buf_free[buf]);
        umma_commit(&s.o_done[t]);
        umma_commit(&s.v_empty[st]);
      }
      for (int j = n; j < n_load && !s.abort; ++j) {
        const int st = j % STAGES;
        if (!wait_or_abort(s, &s.v_full[st], (j / STAGES) & 1)) break;
        mbar_arrive(&s.v_empty[st]);
      }
      umma_commit(&s.drain[t]);
      mbar_wait(&s.drain[t], 0);
    }
  } else {
    regs_increase<SOFTMAX_REGS>();
    const int t = warp / 4;
    softmax_tile<SPLIT>(s, p, tmem, t, warp % 4, lane, bh, qb, q0[t], n_kv[0], n_kv[1], k0, part,
                        parts);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == MMA_WARP) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

// Merge of the partial records of split query blocks: one warp per query row of the split
// blocks (qb >= first_split_qb), lane i owns output features 2i, 2i + 1; lane q also reads part
// q's running max and row sum (at most 32 parts), so the parts' records are fetched in
// parallel. The parts' sums are weighted by exp2(m_part - M) (never averaged outputs);
// O = sum / l, LSE in natural log.
constexpr int COMBINE_WARPS = 8;

__global__ void __launch_bounds__(COMBINE_WARPS * 32)
prefill_combine_kernel(const Params p) {
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int split_blocks = p.n_qblocks - p.first_split_qb;
  const long long g = static_cast<long long>(blockIdx.x) * COMBINE_WARPS + warp;
  const int row_in_block = static_cast<int>(g % BLOCK_M);
  const long long blk = g / BLOCK_M;  // over (bh, split block)
  const int qb = p.first_split_qb + static_cast<int>(blk % split_blocks);
  const int bh = static_cast<int>(blk / split_blocks);
  if (bh >= p.B * p.H) return;  // warp-uniform, as are the two exits below
  const int row = qb * BLOCK_M + row_in_block;
  if (row >= p.Tq) return;
  const int parts = block_parts(p, qb);
  if (parts <= 1) return;
  const float* rec0 = part_record(p, bh, qb, 0, row_in_block);
  const size_t stride = static_cast<size_t>(BLOCK_M) * PART_REC;
  float mq = -INFINITY, lq = 0.f;
  if (lane < parts) {
    const float2 ml = *reinterpret_cast<const float2*>(rec0 + lane * stride + HD);
    mq = ml.x;
    lq = ml.y;
  }
  float M = mq;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  const float w = (mq == -INFINITY) ? 0.f : ex2_approx(mq - M);
  float den = w * lq;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
  float n0 = 0.f, n1 = 0.f;
#pragma unroll 4
  for (int q = 0; q < parts; ++q) {
    const float wq = __shfl_sync(0xffffffffu, w, q);
    const float2 a = reinterpret_cast<const float2*>(rec0 + q * stride)[lane];
    n0 = fmaf(wq, a.x, n0);
    n1 = fmaf(wq, a.y, n1);
  }
  const float inv = den > 0.f ? 1.f / den : 0.f;
  const size_t orow = static_cast<size_t>(bh) * p.Tq + row;
  reinterpret_cast<uint32_t*>(p.o + orow * HD)[lane] = pack_bf16x2(n0 * inv, n1 * inv);
  if (lane == 0) p.lse[orow] = den > 0.f ? (M + log2f(den)) * LN2 : -INFINITY;
}

}  // namespace prefill
}  // namespace tt
