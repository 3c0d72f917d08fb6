// Fused rotary embedding + KV-cache append for one decoder layer (the step that feeds the
// attention in Tiny-transformer's Block.forward, model.py:61-68):
//
//   qkv   [B, T, 3, H, 64] bf16, the fused QKV projection (row-major, as F.linear returns it)
//   q_out [B, H, T, 64]    bf16 contiguous  = rope(q)
//   cache_k[b, h, pos + t] = rope(k),  cache_v[b, h, pos + t] = v      (cache [B, H, C, 64])
//
// RoPE follows reference.py:30-34 operation by operation in bf16: the FP32 cos/sin table
// entries are rounded to bf16, and each product and the final sum / difference are rounded
// to bf16 (round to nearest even), exactly as the reference's bf16 tensor expression
// `even * cos - odd * sin`, `even * sin + odd * cos` evaluates. Pairs are adjacent elements
// (2i, 2i+1) with table column i.
//
// One warp per (b, t, h) row: lane i owns pair i, so every row read and written is one
// coalesced 128-byte access. The start position is either a host value or read from device
// memory (a captured decode step). A position outside the cache or the table is not written:
// the row is skipped and TT_ERR_RANGE is set in the status word.
#pragma once

#include <cuda_bf16.h>

#include "sm100_ptx.cuh"

namespace tt {
namespace rope {

constexpr int HD = 64;
constexpr int PAIRS = HD / 2;
constexpr int ROWS_PER_BLOCK = 8;  // warps per block
constexpr int THREADS = ROWS_PER_BLOCK * 32;

struct Params {
  const __nv_bfloat16* qkv;
  int B, T, H;
  const float* cos;  // [table_len, 32]
  const float* sin;
  long long table_len;
  long long position;            // start position when position_dev is null
  const long long* position_dev;  // optional device-held start position
  __nv_bfloat16* q_out;
  __nv_bfloat16* cache_k;
  __nv_bfloat16* cache_v;
  long long ck_s0, ck_s1, ck_s2;  // element strides of cache_k (batch, head, position)
  long long cv_s0, cv_s1, cv_s2;
  long long capacity;
};

__device__ __forceinline__ float bf16_round(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}

// (e, o) -> (e*c - o*s, e*s + o*c) with bf16 rounding after every operation.
__device__ __forceinline__ uint32_t rotate_pair(uint32_t pair, float c, float s) {
  const float e = bf16_lo(pair);
  const float o = bf16_hi(pair);
  const float r0 = bf16_round(e * c) - bf16_round(o * s);
  const float r1 = bf16_round(e * s) + bf16_round(o * c);
  return pack_bf16x2(r0, r1);
}

__global__ void __launch_bounds__(THREADS) rope_append_kernel(const Params p) {
  const long long row = static_cast<long long>(blockIdx.x) * ROWS_PER_BLOCK + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  const long long rows = static_cast<long long>(p.B) * p.T * p.H;
  if (row >= rows) return;
  const int h = static_cast<int>(row % p.H);
  const long long bt = row / p.H;
  const int t = static_cast<int>(bt % p.T);
  const int b = static_cast<int>(bt / p.T);
  const long long pos = (p.position_dev != nullptr ? *p.position_dev : p.position) + t;
  if (pos < 0 || pos >= p.capacity || pos >= p.table_len) {
    if (lane == 0) atomicOr(&g_tt_status, TT_ERR_RANGE);
    return;
  }
  const float c = bf16_round(p.cos[pos * PAIRS + lane]);
  const float s = bf16_round(p.sin[pos * PAIRS + lane]);

  const uint32_t* src = reinterpret_cast<const uint32_t*>(p.qkv + (bt * 3 * p.H + h) * HD);
  const long long part = static_cast<long long>(p.H) * PAIRS;  // q -> k -> v, in pairs
  const uint32_t qp = src[lane];
  const uint32_t kp = src[part + lane];
  const uint32_t vp = src[2 * part + lane];

  uint32_t* qo = reinterpret_cast<uint32_t*>(
      p.q_out + ((static_cast<long long>(b) * p.H + h) * p.T + t) * HD);
  uint32_t* ko = reinterpret_cast<uint32_t*>(p.cache_k + b * p.ck_s0 + h * p.ck_s1 + pos * p.ck_s2);
  uint32_t* vo = reinterpret_cast<uint32_t*>(p.cache_v + b * p.cv_s0 + h * p.cv_s1 + pos * p.cv_s2);
  qo[lane] = rotate_pair(qp, c, s);
  ko[lane] = rotate_pair(kp, c, s);
  vo[lane] = vp;
}

}  // namespace rope
}  // namespace tt
