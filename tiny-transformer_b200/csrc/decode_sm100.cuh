// Single-token (Tq == 1) KV-cache decode for sm_100a: split-KV with an FP32 LSE combine.
//
// Semantics follow the reference decode path (Tiny-transformer
// csrc/attention/attention_decode_BF16_kernel.cuh:45-128 and reference.py:49-53): the query
// attends to every cached key (Tk == past_len + 1), scale 1/sqrt(64), FP32 softmax, BF16 O,
// natural-log FP32 LSE. Added here: an optional per-sequence valid length kv_lens[b]
// (key j visible iff j < kv_lens[b]); a sequence with no visible key gets O = 0, LSE = -inf,
// the reference's convention for rows without visible keys.
//
// Decode is HBM-bound, so the kernel is built to keep large K/V transfers in flight:
// * work items are (batch*head, chunk of `chunk` keys). A persistent grid of one CTA per SM
//   takes items dynamically from a counter in the workspace (zeroed by the host before the
//   launch), so uneven sequence lengths do not unbalance the SMs;
// * a producer warp streams each item's keys through a STAGES-deep ring of 384-row stages
//   (48 KiB of K + 48 KiB of V) with 1-D bulk async copies (TMA engine, no multicast,
//   evict-first L2 policy), publishing an item header with each stage; rows are read through
//   the cache strides, so prefix views of a larger cache need no copy;
// * 12 consumer warps share each stage, one key row per lane: a lane computes the 64-wide dot
//   product of its row (16-byte shared reads rotated by lane so 32 rows hit distinct banks; q
//   is held pre-rotated in registers), the warp takes one max per 32 rows, and for P.V each
//   lane owns two output features and receives every p by shuffle. Each warp keeps an online
//   softmax (m, l, acc); at the end of an item each warp leaves its (m, l, acc) in a
//   double-buffered shared record and moves on to the next stage;
// * a combine warp merges the 12 records of each item. An item that covers a whole sequence
//   writes O and LSE; otherwise the combine warp writes an FP32 partial (acc[64], m, l),
//   publishes it (release fence, then an arrival on the sequence's counter in the workspace)
//   and, when its arrival is the sequence's last, merges all of the sequence's partials
//   (acquire fence, L2 reads) into O and LSE. The split and the merge are one launch, and the
//   streaming warps never wait for a global-memory round trip.
// Every wait is a bounded mbarrier wait; no CTA waits for another CTA.
#pragma once

#include <cuda_bf16.h>
#include <cstdint>

#include "sm100_ptx.cuh"

namespace tt {
namespace decode {

constexpr int HD = 64;
constexpr int ROW_BYTES = HD * 2;                    // 128 B per key row
constexpr int CONSUMER_WARPS = 12;
constexpr int ROWS_PER_WARP = 32;                    // one key row per lane
constexpr int SUB = CONSUMER_WARPS * ROWS_PER_WARP;  // 384 key rows per ring stage
constexpr int STAGES = 2;
constexpr int STAGE_BYTES = 2 * SUB * ROW_BYTES;     // K then V rows: 96 KiB
constexpr int PRODUCER_WARP = CONSUMER_WARPS;
constexpr int COMBINE_WARP = CONSUMER_WARPS + 1;
constexpr int THREADS = (CONSUMER_WARPS + 2) * 32;
constexpr int MIN_CHUNK = SUB;
constexpr int MAX_CHUNK = 4 * SUB;                   // 1536 keys per work item
constexpr int PARTIAL = HD + 4;                      // acc[64], m (log2 units), l, 2 pad:
                                                     // 272 B records keep float4 stores aligned
constexpr size_t kCounterBytes = 256;                // work counter at the start of the workspace,
                                                     // then (split sequences only) one arrival
                                                     // counter per (batch, head), 256-B rounded
constexpr float LN2 = 0.69314718055994530942f;

struct StageHeader {
  int bh;    // batch * heads + head; -1 ends the stream
  int ch;    // chunk of the item
  int sub;   // stage within the item
  int subs;  // stages in the item
  int rows;  // valid rows of the item
  int nc;    // chunks of this sequence
};

struct ItemHeader {
  int bh;  // batch * heads + head; -1 ends the combine warp's loop
  int ch;  // chunk of the item
  int nc;  // chunks of this sequence
  int pad;
};

struct alignas(128) Smem {
  uint8_t ring[STAGES][STAGE_BYTES];
  float red[2][CONSUMER_WARPS][PARTIAL];  // per-warp item records, double-buffered
  ItemHeader item[2];                     // the item each record buffer holds
  StageHeader hdr[STAGES];
  uint64_t full[STAGES], empty[STAGES];
  uint64_t red_full[2], red_free[2];
  volatile int abort;
};
constexpr size_t kSmemBytes = sizeof(Smem) + 128;

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
  int chunk;                   // keys per work item, multiple of SUB, <= MAX_CHUNK
  int n_chunks;                // ceil(Tk / chunk)
  __nv_bfloat16* o;            // contiguous [B,H,1,64]
  float* lse;                  // [B,H,1]
  unsigned* counter;           // next work item (zero at launch)
  unsigned* arrivals;          // [B*H] partials written per sequence (zero at launch; used
                               // when n_chunks > 1)
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

__device__ __forceinline__ void unpack_row8(const uint4 u, float (&f)[8]) {
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x);
  f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z);
  f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}

// Bounded wait that also gives up once another warp of the CTA has aborted.
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

__device__ __forceinline__ bool warp_wait(Smem& s, uint64_t* bar, uint32_t parity) {
  return __all_sync(0xffffffffu, wait_or_abort(s, bar, parity));
}

// Ring position: stage index and the parity of its current use.
struct Ring {
  int st = 0;
  uint32_t ph = 0;
  int used = 0;  // stages handed out so far (saturating at STAGES)
  __device__ __forceinline__ void next() {
    if (++st == STAGES) {
      st = 0;
      ph ^= 1u;
    }
    if (used < STAGES) ++used;
  }
};

__device__ __forceinline__ unsigned grab(const Params& p, int lane) {
  unsigned i = 0;
  if (lane == 0) i = atomicAdd(p.counter, 1u);
  return __shfl_sync(0xffffffffu, i, 0);
}

// Producer warp: take items from the counter and stream their K and V rows into the ring,
// each stage with its header; a final header with bh = -1 ends the consumers' loop.
__device__ __forceinline__ void produce(Smem& s, const Params& p, int lane) {
  const uint64_t pol = l2_policy_evict_first();
  const unsigned total = static_cast<unsigned>(p.B * p.H * p.n_chunks);
  Ring r;
  uint32_t armed = 0;             // bit i: stage i has been armed at least once
  uint32_t armed_ph = 0;          // bit i: parity of stage i's last armed phase
  unsigned item = grab(p, lane);
  bool ok = true;
  while (ok && item < total) {
    const unsigned next_item = grab(p, lane);  // overlap the atomic with this item's copies
    const int bh = static_cast<int>(item / static_cast<unsigned>(p.n_chunks));
    const int ch = static_cast<int>(item - static_cast<unsigned>(bh) * p.n_chunks);
    const int L = valid_len(p, bh / p.H);
    const int nc = chunks_for(L, p.chunk);
    if (ch < nc) {
      const int rows = max(0, min(p.chunk, L - ch * p.chunk));
      const int subs = rows == 0 ? 1 : (rows + SUB - 1) / SUB;
      const int b = bh / p.H, h = bh - b * p.H;
      for (int sub = 0; sub < subs; ++sub) {
        if (r.used == STAGES && !warp_wait(s, &s.empty[r.st], r.ph ^ 1u)) { ok = false; break; }
        const int rs = max(0, min(SUB, rows - sub * SUB));
        if (lane == 0) {
          s.hdr[r.st] = StageHeader{bh, ch, sub, subs, rows, nc};
          mbar_arrive_expect_tx(&s.full[r.st], static_cast<uint32_t>(2 * rs * ROW_BYTES));
        }
        armed |= 1u << r.st;
        armed_ph = (armed_ph & ~(1u << r.st)) | (r.ph << r.st);
        if (rs > 0) {
          __syncwarp();
          const int64_t key0 = static_cast<int64_t>(ch) * p.chunk + sub * SUB;
          const __nv_bfloat16* kb = p.k + b * p.k_sb + h * p.k_sh + key0 * p.k_st;
          const __nv_bfloat16* vb = p.v + b * p.v_sb + h * p.v_sh + key0 * p.v_st;
          uint8_t* ks = s.ring[r.st];
          uint8_t* vs = s.ring[r.st] + SUB * ROW_BYTES;
          if (p.k_st == HD && p.v_st == HD) {
            if (lane == 0) {
              bulk_load(ks, kb, rs * ROW_BYTES, &s.full[r.st], pol);
              bulk_load(vs, vb, rs * ROW_BYTES, &s.full[r.st], pol);
            }
          } else {
            // Strided rows (16-byte aligned): one 128-byte copy per row and tensor.
            for (int i = lane; i < rs; i += 32) {
              bulk_load(ks + i * ROW_BYTES, kb + i * p.k_st, ROW_BYTES, &s.full[r.st], pol);
              bulk_load(vs + i * ROW_BYTES, vb + i * p.v_st, ROW_BYTES, &s.full[r.st], pol);
            }
          }
        }
        r.next();
      }
    }
    item = next_item;
  }
  // End of stream: a header with bh = -1 in the next stage.
  if (ok && (r.used < STAGES || warp_wait(s, &s.empty[r.st], r.ph ^ 1u))) {
    if (lane == 0) {
      s.hdr[r.st].bh = -1;
      mbar_arrive_expect_tx(&s.full[r.st], 0);
    }
  }
  // On abort, wait (bounded) for the last armed phase of every stage, so the CTA never
  // retires while a bulk copy into its shared memory is pending.
  if (s.abort && lane == 0) {
    for (int i = 0; i < STAGES; ++i)
      if (armed & (1u << i)) mbar_wait(&s.full[i], (armed_ph >> i) & 1u);
  }
}

// Merge all partials of sequence bh (called by one warp once every chunk's partial is
// published): lane c reads chunk c's (m, l), the warp reduces the max, and each lane accumulates
// two features over all chunks with the weights exp2(m_c - M) broadcast by shuffle (never
// averages normalised outputs). The partials were written by other SMs, so they are read from
// L2 (ld.global.cg), not through this SM's L1.
__device__ __forceinline__ void merge_sequence(const Params& p, int bh, int nc, int lane) {
  const float* src = p.partials + static_cast<size_t>(bh) * p.n_chunks * PARTIAL;
  float M = -INFINITY;
  for (int c = lane; c < nc; c += 32) M = fmaxf(M, __ldcg(src + c * PARTIAL + HD));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float n0 = 0.f, n1 = 0.f, den = 0.f;
  for (int base = 0; base < nc; base += 32) {
    const int c = base + lane;
    float w = 0.f;
    if (c < nc) {
      const float mc = __ldcg(src + c * PARTIAL + HD);
      w = (mc == -INFINITY) ? 0.f : ex2_approx(mc - M);
      den = fmaf(w, __ldcg(src + c * PARTIAL + HD + 1), den);
    }
    const int cnt = min(32, nc - base);
#pragma unroll 4
    for (int i = 0; i < cnt; ++i) {
      const float wi = __shfl_sync(0xffffffffu, w, i);
      const float2 a = __ldcg(reinterpret_cast<const float2*>(src + (base + i) * PARTIAL) + lane);
      n0 = fmaf(wi, a.x, n0);
      n1 = fmaf(wi, a.y, n1);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) den += __shfl_xor_sync(0xffffffffu, den, off);
  const float inv = den > 0.f ? 1.f / den : 0.f;
  reinterpret_cast<uint32_t*>(p.o + static_cast<size_t>(bh) * HD)[lane] =
      pack_bf16x2(n0 * inv, n1 * inv);
  if (lane == 0) p.lse[bh] = den > 0.f ? (M + log2f(den)) * LN2 : -INFINITY;
}

// Combine warp: for each item, merge the CONSUMER_WARPS warp records (lane t owns features
// 2t, 2t + 1), free the record buffer, then write O and LSE (whole sequence) or the item's
// partial. A partial is published with a release fence before the arrival on the sequence's
// counter; the warp whose arrival completes the count takes an acquire fence and merges the
// sequence. Nothing here waits on another CTA.
__device__ __forceinline__ void combine_items(Smem& s, const Params& p, int lane) {
  unsigned items = 0;
  while (true) {
    const int buf = static_cast<int>(items & 1u);
    const uint32_t use = items >> 1;
    if (!warp_wait(s, &s.red_full[buf], use & 1)) break;
    const ItemHeader it = s.item[buf];
    if (it.bh < 0) break;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < CONSUMER_WARPS; ++w) M = fmaxf(M, s.red[buf][w][HD]);
    float n0 = 0.f, n1 = 0.f, den = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < CONSUMER_WARPS; ++w) {
        const float mw = s.red[buf][w][HD];
        if (mw == -INFINITY) continue;
        const float wt = ex2_approx(mw - M);
        const float2 a = reinterpret_cast<const float2*>(s.red[buf][w])[lane];
        n0 = fmaf(wt, a.x, n0);
        n1 = fmaf(wt, a.y, n1);
        den = fmaf(wt, s.red[buf][w][HD + 1], den);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&s.red_free[buf]);
    ++items;
    if (it.nc == 1) {
      const float inv = den > 0.f ? 1.f / den : 0.f;
      reinterpret_cast<uint32_t*>(p.o + static_cast<size_t>(it.bh) * HD)[lane] =
          pack_bf16x2(n0 * inv, n1 * inv);
      if (lane == 0) p.lse[it.bh] = den > 0.f ? (M + log2f(den)) * LN2 : -INFINITY;
      continue;
    }
    float* dst = p.partials + (static_cast<size_t>(it.bh) * p.n_chunks + it.ch) * PARTIAL;
    reinterpret_cast<float2*>(dst)[lane] = make_float2(n0, n1);
    if (lane == 0) {
      dst[HD] = M;
      dst[HD + 1] = den;
    }
    // Release: every lane's partial stores are ordered before the arrival.
    __threadfence();
    __syncwarp();
    unsigned arrived = 0;
    if (lane == 0) arrived = atomicAdd(p.arrivals + it.bh, 1u);
    arrived = __shfl_sync(0xffffffffu, arrived, 0);
    if (arrived + 1 == static_cast<unsigned>(it.nc)) {
      // Acquire: the other chunks' partials, published before their arrivals, are visible.
      __threadfence();
      merge_sequence(p, it.bh, it.nc, lane);
    }
  }
}

__global__ void __launch_bounds__(THREADS, 1)
decode_split_kernel(const Params p) {
  extern __shared__ uint8_t smem_raw[];
  Smem& s = *reinterpret_cast<Smem*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) &
                                     ~uintptr_t(127));
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&s.full[i], 1);
      mbar_init(&s.empty[i], CONSUMER_WARPS);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s.red_full[i], CONSUMER_WARPS);
      mbar_init(&s.red_free[i], 1);
    }
    s.abort = 0;
    fence_barrier_init();
  }
  __syncthreads();

  if (warp == PRODUCER_WARP) {
    produce(s, p, lane);
  } else if (warp < CONSUMER_WARPS) {
    const int row0 = warp * ROWS_PER_WARP;
    Ring r;
    unsigned items = 0;    // items finished by this CTA
    float qr[8][8];        // q * scale * log2(e); 16-byte chunk (cc + lane) & 7 in qr[cc]
    float m = -INFINITY;   // warp-uniform running max (log2 units)
    float l = 0.f;         // this lane's share of the running sum
    float a0 = 0.f, a1 = 0.f;  // output features 2*lane, 2*lane + 1
    bool ended = false;    // saw the producer's end-of-stream header
    while (true) {
      if (!warp_wait(s, &s.full[r.st], r.ph)) break;
      const StageHeader hd = s.hdr[r.st];
      if (hd.bh < 0) {
        ended = true;
        break;
      }
      if (hd.sub == 0) {
        // New item: rotated q and a fresh online softmax.
        const int b = hd.bh / p.H, h = hd.bh - b * p.H;
        const uint8_t* qrow = reinterpret_cast<const uint8_t*>(p.q + b * p.q_sb + h * p.q_sh);
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          unpack_row8(*reinterpret_cast<const uint4*>(qrow + ((cc + lane) & 7) * 16), qr[cc]);
#pragma unroll
          for (int e = 0; e < 8; ++e) qr[cc][e] *= p.scale_log2;
        }
        m = -INFINITY;
        l = 0.f;
        a0 = a1 = 0.f;
      }
      // Ring reads use explicit shared-memory loads (ld.shared): through the re-aligned Smem
      // pointer the compiler would emit generic loads, measured 3.6 % slower on cfg4.
      const uint32_t ks = smem_u32(s.ring[r.st]) + row0 * ROW_BYTES;
      const uint32_t vs = smem_u32(s.ring[r.st]) + (SUB + row0) * ROW_BYTES;
      const int r_valid = max(0, min(SUB, hd.rows - hd.sub * SUB)) - row0;  // this warp's rows

      float x = -INFINITY;  // score of this lane's row
      if (lane < r_valid) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int cc = 0; cc < 8; ++cc) {
          float kf[8];
          unpack_row8(lds_u4(ks + lane * ROW_BYTES + ((cc + lane) & 7) * 16), kf);
#pragma unroll
          for (int e = 0; e < 8; ++e) d[e & 3] = fmaf(qr[cc][e], kf[e], d[e & 3]);
        }
        x = (d[0] + d[1]) + (d[2] + d[3]);
      }
      float mx = x;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float m_new = fmaxf(m, mx);
      if (m_new != -INFINITY) {  // warp-uniform
        const float f = ex2_approx(m - m_new);   // m == -inf -> 0
        const float pr = ex2_approx(x - m_new);  // invalid rows: exp2(-inf) = 0
        l = l * f + pr;
        float b0[4] = {a0 * f, 0.f, 0.f, 0.f}, b1[4] = {a1 * f, 0.f, 0.f, 0.f};
        const uint32_t vcol = vs + lane * 4;
        if (r_valid >= ROWS_PER_WARP) {
#pragma unroll
          for (int rr = 0; rr < ROWS_PER_WARP; ++rr) {
            const float pb = __shfl_sync(0xffffffffu, pr, rr);
            const uint32_t vv = lds_u32(vcol + rr * ROW_BYTES);
            b0[rr & 3] = fmaf(pb, bf16_lo(vv), b0[rr & 3]);
            b1[rr & 3] = fmaf(pb, bf16_hi(vv), b1[rr & 3]);
          }
        } else {
          // Tail of a sequence: the same loop under a warp-uniform guard (unrolled, so the
          // accumulator indices stay static and in registers).
#pragma unroll
          for (int rr = 0; rr < ROWS_PER_WARP; ++rr) {
            if (rr < r_valid) {
              const float pb = __shfl_sync(0xffffffffu, pr, rr);
              const uint32_t vv = lds_u32(vcol + rr * ROW_BYTES);
              b0[rr & 3] = fmaf(pb, bf16_lo(vv), b0[rr & 3]);
              b1[rr & 3] = fmaf(pb, bf16_hi(vv), b1[rr & 3]);
            }
          }
        }
        a0 = (b0[0] + b0[1]) + (b0[2] + b0[3]);
        a1 = (b1[0] + b1[1]) + (b1[2] + b1[3]);
        m = m_new;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&s.empty[r.st]);  // this warp is done reading the stage
      r.next();

      if (hd.sub + 1 == hd.subs) {
        // End of item: this warp's record (m, l, acc[64]) into a double-buffered shared slot
        // for the combine warp.
        float lsum = l;
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
        const int buf = static_cast<int>(items & 1u);
        const uint32_t use = items >> 1;
        if (use > 0 && !warp_wait(s, &s.red_free[buf], (use - 1) & 1)) break;
        float* rec = s.red[buf][warp];
        reinterpret_cast<float2*>(rec)[lane] = make_float2(a0, a1);
        if (lane == 0) {
          rec[HD] = m;
          rec[HD + 1] = lsum;
          if (warp == 0) s.item[buf] = ItemHeader{hd.bh, hd.ch, hd.nc, 0};
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&s.red_full[buf]);
        ++items;
      }
    }
    if (ended) {
      // End of stream for the combine warp: an item header with bh = -1.
      const int buf = static_cast<int>(items & 1u);
      const uint32_t use = items >> 1;
      if (use == 0 || warp_wait(s, &s.red_free[buf], (use - 1) & 1)) {
        if (lane == 0) {
          if (warp == 0) s.item[buf].bh = -1;
          mbar_arrive(&s.red_full[buf]);
        }
      }
    }
  } else {
    combine_items(s, p, lane);
  }
  __syncthreads();
}

}  // namespace decode
}  // namespace tt
