// C-ABI implementation (include/tt_attention.h): argument validation, path selection
// (split-KV decode for q_len == 1, tcgen05 prefill otherwise), TMA descriptor encoding
// and kernel launches on the caller's stream. Nothing here allocates device memory.
//
// Reference host dispatcher this replaces: Tiny-transformer csrc/attention/attention.cu:32-159.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>
#include <string>

#include "tt_attention.h"
#include "sm100_ptx.cuh"
#include "prefill_sm100.cuh"
#include "decode_sm100.cuh"
#include "decode_direct_sm100.cuh"
#include "selftest_sm100.cuh"
#include "rope_append_sm100.cuh"
#include "qkv_rope_sm100.cuh"
#include "backward_sm100.cuh"
#include "backward_det_sm100.cuh"

namespace {

constexpr float kScaleLog2 = 0.125f * 1.44269504088896340736f;  // (1/sqrt(64)) * log2(e)
constexpr int kMaxDevices = 64;

thread_local std::string g_last_error;

tt_attn_status fail(tt_attn_status st, const std::string& msg) {
  g_last_error = msg;
  return st;
}

// ------------------------------------------------------------------ shape helpers
struct Shape4 {
  int64_t size[4];
  int64_t stride[4];
};

// Strides of size-1 dimensions are never used to address memory; give them the
// canonical contiguous value so stride checks and TMA descriptors accept them.
Shape4 canonical(int64_t b, int64_t h, int64_t t, const int64_t* strides) {
  Shape4 s{{b, h, t, TT_ATTN_HEAD_DIM}, {strides[0], strides[1], strides[2], strides[3]}};
  const int64_t contiguous[3] = {h * t * TT_ATTN_HEAD_DIM, t * TT_ATTN_HEAD_DIM, TT_ATTN_HEAD_DIM};
  for (int d = 0; d < 3; ++d)
    if (s.size[d] == 1) s.stride[d] = contiguous[d];
  return s;
}

bool strides_ok(const int64_t* st) {
  if (st[3] != 1) return false;
  for (int d = 0; d < 3; ++d)
    if (st[d] <= 0 || st[d] % 8 != 0) return false;
  return true;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Keys per decode work item: MAX_CHUNK halved (never below MIN_CHUNK; every value is a multiple
// of the ring stage) until the shape gives about 8 items per CTA of a persistent grid on a
// 148-SM part, for load balance (a shape-only heuristic, so the workspace size does not depend
// on the device).
int decode_chunk(int64_t bh, int64_t tk) {
  constexpr int64_t kTargetItems = 8 * 148;
  int chunk = tt::decode::MAX_CHUNK;
  while (chunk > tt::decode::MIN_CHUNK && bh * ((tk + chunk - 1) / chunk) < kTargetItems)
    chunk /= 2;
  return chunk;
}

// Decode path choice (shape only, so the workspace size never depends on the device): the
// cluster kernel (decode_direct_sm100.cuh: no workspace, one launch, <= 4 CTAs per sequence)
// up to 2^20 (batch * heads * kv_len) K/V rows (256 MB), and up to 2^21 rows when there are at
// most 640 (batch, head) sequences; the persistent split-KV kernel (decode_sm100.cuh: dynamic
// work items balance uneven kv_lens) above. Measured with the L2 flushed, full lengths / kv_lens
// U[Tk/8, Tk]: 1.57M rows as 192 sequences of 8192 keys 82.9 / 60.4 us against 96.3 / 69.5 in
// the persistent kernel, 1.18M rows as 576 sequences 68.5 / 48.2 against 73.7 / 55.3, but 1.57M
// rows as 768 or 1536 sequences 80-81 / 58 against 78-80 / 55-57; 3.1M rows (384 sequences,
// kv_lens) 98 against 90. Few long sequences ran at 1.6-2.5 TB/s in the persistent kernel, so
// there is no separate key-count limit.
constexpr int64_t kDirectDecodeMaxRows = int64_t(1) << 20;
constexpr int64_t kDirectDecodeFewSeqMaxRows = int64_t(1) << 21;
constexpr int64_t kDirectDecodeFewSeq = 640;

constexpr int64_t kDirectDecodeMaxSplits = 4;

bool use_direct_decode(int64_t bh, int64_t kv_len) {
  const int64_t rows = bh * kv_len;
  return rows <= kDirectDecodeMaxRows ||
         (bh <= kDirectDecodeFewSeq && rows <= kDirectDecodeFewSeqMaxRows);
}

// Prefill work plan (shape only, so the workspace size never depends on the device). A CTA
// computes one 256-row query block over its causal KV range, heaviest blocks first. When the
// grid has fewer blocks than a 148-SM part has SMs, the longest block's KV loop sets the
// kernel time (one long sequence, or few (batch x head) rows per GPU). The plan then splits
// blocks longer than part_tiles into near-equal parts (separate CTAs, merged by
// prefill_combine_kernel), with the smallest part_tiles (at least 4 KV tiles) whose CTAs
// still fit one wave of 148. With more blocks than SMs no split is made: a second wave of
// short CTAs measured slower than the unsplit grid (each CTA's prologue and epilogue cost
// about three KV steps, and the combine kernel two).
constexpr int64_t kPlanSms = 148;
constexpr int64_t kMinPartTiles = 4;
constexpr int kMaxParts = 32;  // prefill_combine_kernel reads one part per lane

struct PrefillPlan {
  int part_tiles = 0;  // 0: no split
  int max_parts = 1;
  int first_split_qb = 0;
  int64_t ctas = 0;
};

int64_t host_kv_tiles(int64_t tq, int64_t tk, int64_t past, int64_t q0) {
  if (q0 >= tq) return 0;
  const int64_t end = std::min(tk, q0 + tt::prefill::BM + past);
  return (end + tt::prefill::BN - 1) / tt::prefill::BN;
}

int64_t host_block_tiles(int64_t tq, int64_t tk, int64_t past, int64_t qb) {
  const int64_t q0 = qb * tt::prefill::BLOCK_M;
  return std::max(host_kv_tiles(tq, tk, past, q0),
                  host_kv_tiles(tq, tk, past, q0 + tt::prefill::BM));
}

PrefillPlan prefill_plan(int64_t bh, int64_t tq, int64_t tk, int64_t past) {
  PrefillPlan pl;
  const int64_t nqb = (tq + tt::prefill::BLOCK_M - 1) / tt::prefill::BLOCK_M;
  pl.ctas = bh * nqb;
  if (pl.ctas >= kPlanSms) return pl;
  const int64_t longest = host_block_tiles(tq, tk, past, nqb - 1);  // never decreases with qb
  for (int64_t part = kMinPartTiles; part < longest; ++part) {
    if ((longest + part - 1) / part > kMaxParts) continue;
    int64_t ctas = 0;
    for (int64_t qb = 0; qb < nqb; ++qb)
      ctas += std::max<int64_t>(1, (host_block_tiles(tq, tk, past, qb) + part - 1) / part);
    if (ctas * bh > kPlanSms) continue;
    pl.part_tiles = static_cast<int>(part);
    pl.max_parts = static_cast<int>((longest + part - 1) / part);
    pl.ctas = ctas * bh;
    pl.first_split_qb = static_cast<int>(nqb);
    for (int64_t qb = nqb - 1; qb >= 0 && host_block_tiles(tq, tk, past, qb) > part; --qb)
      pl.first_split_qb = static_cast<int>(qb);
    return pl;
  }
  return pl;  // no part size fits one wave (or the blocks are already short): no split
}

size_t prefill_workspace_bytes(int64_t bh, int64_t tq, const PrefillPlan& pl) {
  if (pl.part_tiles == 0) return 0;
  const int64_t nqb = (tq + tt::prefill::BLOCK_M - 1) / tt::prefill::BLOCK_M;
  return static_cast<size_t>(bh * nqb * pl.max_parts) * tt::prefill::BLOCK_M *
         tt::prefill::PART_REC * sizeof(float);
}

// Bytes of the per-sequence arrival counters of a split decode (one unsigned per (batch, head),
// rounded up to 256 bytes so the partials after them stay aligned).
size_t decode_arrival_bytes(int64_t bh) {
  return (static_cast<size_t>(bh) * sizeof(unsigned) + 255) & ~size_t(255);
}

// ------------------------------------------------------------------ driver entry point
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// 4-D map over [B, H, T, 64] bf16 (dims listed innermost first), box 64 x box_rows rows,
// 128-byte swizzle; rows past T read as zero.
bool encode_map(CUtensorMap* map, const void* base, const Shape4& s, std::string* err,
                unsigned box_rows = tt::prefill::BM) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is not available from the CUDA driver";
    return false;
  }
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(s.size[3]), static_cast<cuuint64_t>(s.size[2]),
                              static_cast<cuuint64_t>(s.size[1]), static_cast<cuuint64_t>(s.size[0])};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(s.stride[2]) * 2,
                                 static_cast<cuuint64_t>(s.stride[1]) * 2,
                                 static_cast<cuuint64_t>(s.stride[0]) * 2};
  const cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
    *err = buf;
    return false;
  }
  return true;
}

// FP32 [B, H, T, 64] map for the backward's dQ accumulator: boxes of 32 features (128 bytes,
// 128-byte swizzle) x box_rows rows, written by bulk tensor reduce-add.
bool encode_map_f32(CUtensorMap* map, void* base, const Shape4& s, std::string* err,
                    unsigned box_rows) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is not available from the CUDA driver";
    return false;
  }
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(s.size[3]), static_cast<cuuint64_t>(s.size[2]),
                              static_cast<cuuint64_t>(s.size[1]), static_cast<cuuint64_t>(s.size[0])};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(s.stride[2]) * 4,
                                 static_cast<cuuint64_t>(s.stride[1]) * 4,
                                 static_cast<cuuint64_t>(s.stride[0]) * 4};
  const cuuint32_t box[4] = {32, static_cast<cuuint32_t>(box_rows), 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, base, dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
    *err = buf;
    return false;
  }
  return true;
}

// 2-D map over a row-major [rows, cols] bf16 matrix (dims innermost first), box 64 x 128,
// 128-byte swizzle; rows past `rows` read as zero. cols * 2 must be a multiple of 16 bytes.
bool encode_map_2d(CUtensorMap* map, const void* base, int64_t rows, int64_t cols,
                   uint32_t box_rows, std::string* err) {
  EncodeTiledFn fn = encode_tiled_fn();
  if (!fn) {
    *err = "cuTensorMapEncodeTiled is not available from the CUDA driver";
    return false;
  }
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[96];
    std::snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (CUresult %d)", int(r));
    *err = buf;
    return false;
  }
  return true;
}


// Launch plan of the fused QKV kernel.
// One row tile (B * T <= 128): split-K clusters. Per feature-tile width (64, 32, 16, widest
// first) the largest K split S <= 3 (at most one part per K slice) whose clusters are all
// resident at once (cudaOccupancyMaxActiveClusters: clusters of S CTAs fit per GPC, so S = 4
// with 36 tiles already needs a second wave on 148 SMs); the first width whose grid covers 70 %
// of the SMs is taken, else the widest grid. The partial sums of all parts meet in rank 0's
// shared memory, and that reduction grows with S: on the decode shapes (B = 1..32, H = 12,
// 768 features) 64-feature tiles x 3 parts measured fastest (4.7-5.2 us against 5.1-13.9 for
// 2, 4, 6 or 8 parts and for 32- or 16-feature tiles).
// More rows: the persistent kernel over 128-feature tiles (64 with an odd head count, so that a
// tile stays inside one of q, k, v), one CTA per SM.
struct QkvRopePlan {
  bool splitk = false;
  int bn = 0;
  int splits = 1;
  int64_t n_tiles = 0, m_tiles = 0;
  int red_rows = 0;
  unsigned grid = 0;
  size_t smem = 0;
};

size_t qkv_splitk_fixed(int bn) {
  namespace qr = tt::qkv_rope;
  return bn == 64 ? qr::splitk_fixed_bytes<64>()
                  : bn == 32 ? qr::splitk_fixed_bytes<32>() : qr::splitk_fixed_bytes<16>();
}

constexpr size_t kMaxDynamicSmem = 227 * 1024;
constexpr int kQkvMaxSplits = 3;

// Clusters of `splits` split-K CTAs (feature tile bn, `smem` bytes each) resident at once on
// the current device; cached, since every decode step asks.
int qkv_max_clusters(int dev, int bn, int splits, size_t smem) {
  namespace qr = tt::qkv_rope;
  struct Key { int dev, bn, splits; size_t smem; int n; };
  static std::mutex mu;
  static std::vector<Key> cache;
  {
    std::lock_guard<std::mutex> lock(mu);
    for (const Key& k : cache)
      if (k.dev == dev && k.bn == bn && k.splits == splits && k.smem == smem) return k.n;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(splits), 1, 1);
  cfg.blockDim = dim3(qr::THREADS, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e;
  if (bn == 64) e = cudaOccupancyMaxActiveClusters(&n, qr::qkv_rope_splitk_kernel<64>, &cfg);
  else if (bn == 32) e = cudaOccupancyMaxActiveClusters(&n, qr::qkv_rope_splitk_kernel<32>, &cfg);
  else e = cudaOccupancyMaxActiveClusters(&n, qr::qkv_rope_splitk_kernel<16>, &cfg);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    n = 0;  // unknown: treated as "does not fit", so only S = 1 is taken
  }
  std::lock_guard<std::mutex> lock(mu);
  if (cache.size() < 256) cache.push_back({dev, bn, splits, smem, n});
  return n;
}

QkvRopePlan qkv_rope_plan(int64_t rows, int64_t heads, int64_t dim, int dev, int sms) {
  namespace qr = tt::qkv_rope;
  QkvRopePlan pl;
  const int64_t n = 3 * heads * TT_ATTN_HEAD_DIM;
  const int64_t n_k = dim / qr::BK;
  const int64_t sm = sms > 0 ? sms : 148;
  pl.m_tiles = (rows + qr::BM - 1) / qr::BM;
  if (pl.m_tiles == 1) {
    pl.splitk = true;
    pl.red_rows = static_cast<int>((rows + 7) / 8 * 8);
    const int64_t want = (sm * 70 + 99) / 100;
    QkvRopePlan best = pl;
    for (int bn : {64, 32, 16}) {
      const int64_t tiles = n / bn;
      auto bytes = [&](int64_t k) {  // fixed part + k partial-sum buffers [rows][bn + 4]
        return qkv_splitk_fixed(bn) + static_cast<size_t>(k) * (bn + 4) * pl.red_rows * 4;
      };
      int64_t sp = 1;
      for (int64_t k = 2; k <= std::min<int64_t>(kQkvMaxSplits, n_k); ++k)
        if (bytes(k) <= kMaxDynamicSmem &&
            tiles <= qkv_max_clusters(dev, bn, static_cast<int>(k), bytes(k)))
          sp = k;
      QkvRopePlan c = pl;
      c.bn = bn;
      c.splits = static_cast<int>(sp);
      c.n_tiles = tiles;
      c.grid = static_cast<unsigned>(tiles * sp);
      c.smem = bytes(sp);
      if (best.bn == 0 || c.grid > best.grid) best = c;
      if (tiles * sp >= want) return c;
    }
    return best;
  }
  pl.bn = heads % 2 == 0 ? 128 : 64;
  pl.n_tiles = n / pl.bn;
  pl.grid = static_cast<unsigned>(std::min<int64_t>(pl.m_tiles * pl.n_tiles, sm));
  pl.smem = pl.bn == 128 ? qr::persistent_smem_bytes<128>() : qr::persistent_smem_bytes<64>();
  return pl;
}

cudaError_t launch_qkv_rope(const QkvRopePlan& pl, const CUtensorMap& tm_h, const CUtensorMap& tm_w,
                            const tt::qkv_rope::Params& p, cudaStream_t stream) {
  namespace qr = tt::qkv_rope;
  if (!pl.splitk) {
    if (pl.bn == 128)
      qr::qkv_rope_persistent_kernel<128><<<pl.grid, qr::THREADS, pl.smem, stream>>>(tm_h, tm_w, p);
    else
      qr::qkv_rope_persistent_kernel<64><<<pl.grid, qr::THREADS, pl.smem, stream>>>(tm_h, tm_w, p);
    return cudaSuccess;
  }
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(pl.splits), static_cast<unsigned>(pl.n_tiles), 1);
  cfg.blockDim = dim3(qr::THREADS, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(pl.splits);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (pl.bn == 64) return cudaLaunchKernelEx(&cfg, qr::qkv_rope_splitk_kernel<64>, tm_h, tm_w, p);
  if (pl.bn == 32) return cudaLaunchKernelEx(&cfg, qr::qkv_rope_splitk_kernel<32>, tm_h, tm_w, p);
  return cudaLaunchKernelEx(&cfg, qr::qkv_rope_splitk_kernel<16>, tm_h, tm_w, p);
}

cudaError_t set_qkv_rope_attributes() {
  namespace qr = tt::qkv_rope;
  const int split_max = static_cast<int>(kMaxDynamicSmem);
  cudaError_t e = cudaFuncSetAttribute(qr::qkv_rope_persistent_kernel<128>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(qr::persistent_smem_bytes<128>()));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qr::qkv_rope_persistent_kernel<64>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(qr::persistent_smem_bytes<64>()));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qr::qkv_rope_splitk_kernel<64>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, split_max);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qr::qkv_rope_splitk_kernel<32>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, split_max);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(qr::qkv_rope_splitk_kernel<16>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, split_max);
  return e;
}

// ------------------------------------------------------------------ per-device setup
struct DeviceState {
  bool checked = false;
  bool supported = false;
  bool attrs_set = false;
  int sm_count = 0;
};
DeviceState g_dev[kMaxDevices];
std::mutex g_dev_mu;

tt_attn_status prepare_device(int* dev_out, int* sm_count = nullptr) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(TT_ATTN_LAUNCH_FAIL, std::string("cudaGetDevice: ") + cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(TT_ATTN_UNSUPPORTED, "device index out of range");
  // Make the device's primary context current on this thread: a thread that has made no
  // runtime call yet (e.g. an autograd worker) has none, and the driver-API tensor-map
  // encoding that follows needs one.
  e = cudaSetDevice(dev);
  if (e != cudaSuccess) return fail(TT_ATTN_LAUNCH_FAIL, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  *dev_out = dev;
  std::lock_guard<std::mutex> lock(g_dev_mu);
  DeviceState& ds = g_dev[dev];
  if (!ds.checked) {
    int major = 0, minor = 0;
    e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (e != cudaSuccess)
      return fail(TT_ATTN_LAUNCH_FAIL, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
    ds.supported = (major == 10);
    e = cudaDeviceGetAttribute(&ds.sm_count, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess)
      return fail(TT_ATTN_LAUNCH_FAIL, std::string("cudaDeviceGetAttribute: ") + cudaGetErrorString(e));
    ds.checked = true;
    if (!ds.supported) {
      char buf[160];
      std::snprintf(buf, sizeof(buf),
                    "bf16 attention kernels require an sm_100 GPU (compute capability 10.x); "
                    "device %d is SM%d%d",
                    dev, major, minor);
      g_last_error = buf;
    }
  }
  if (!ds.supported) {
    char buf[96];
    std::snprintf(buf, sizeof(buf),
                  "bf16 attention kernels require an sm_100 GPU (compute capability 10.x)");
    return fail(TT_ATTN_UNSUPPORTED, buf);
  }
  if (!ds.attrs_set) {
    // The prefill kernel hands registers between warpgroups (setmaxnreg); that is only
    // sound when it launches with exactly the register count the hand-over was sized for.
    const void* prefill_fns[2] = {
        reinterpret_cast<const void*>(tt::prefill::attention_prefill_kernel<false>),
        reinterpret_cast<const void*>(tt::prefill::attention_prefill_kernel<true>)};
    const unsigned launch_regs = tt::prefill::LAUNCH_REGS;
    const int prefill_smem = static_cast<int>(tt::prefill::kSmemBytes);
    for (const void* prefill_fn : prefill_fns) {
      cudaFuncAttributes fa{};
      e = cudaFuncGetAttributes(&fa, prefill_fn);
      if (e != cudaSuccess)
        return fail(TT_ATTN_LAUNCH_FAIL,
                    std::string("cudaFuncGetAttributes: ") + cudaGetErrorString(e));
      if (fa.numRegs != static_cast<int>(launch_regs)) {
        char buf[160];
        std::snprintf(buf, sizeof(buf),
                      "prefill kernel was compiled with %d registers per thread, expected %u; "
                      "rebuild libtt_attention.so",
                      fa.numRegs, launch_regs);
        return fail(TT_ATTN_UNSUPPORTED, buf);
      }
      e = cudaFuncSetAttribute(prefill_fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               prefill_smem);
      if (e != cudaSuccess) break;
    }
    if (e == cudaSuccess) e = set_qkv_rope_attributes();
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tt::decode_direct::decode_direct_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tt::decode_direct::kSmemBytes));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tt::decode::decode_split_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tt::decode::kSmemBytes));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tt::backward::fused::bwd_fused_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tt::backward::fused::kSmemBytes));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tt::backward_det::bwd_dq_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tt::backward_det::kSmemQ));
    if (e == cudaSuccess)
      e = cudaFuncSetAttribute(tt::backward_det::bwd_dkdv_kernel,
                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                               static_cast<int>(tt::backward_det::kSmemKV));
    if (e != cudaSuccess)
      return fail(TT_ATTN_LAUNCH_FAIL, std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    ds.attrs_set = true;
  }
  if (sm_count) *sm_count = ds.sm_count;
  return TT_ATTN_OK;
}

tt_attn_status check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(TT_ATTN_LAUNCH_FAIL, std::string(what) + ": " + cudaGetErrorString(e));
  return TT_ATTN_OK;
}

}  // namespace

extern "C" {

TT_ATTN_API int tt_attn_abi_version(void) { return TT_ATTN_ABI_VERSION; }

TT_ATTN_API const char* tt_attn_status_string(tt_attn_status status) {
  switch (status) {
    case TT_ATTN_OK: return "TT_ATTN_OK";
    case TT_ATTN_BAD_ARG: return "TT_ATTN_BAD_ARG";
    case TT_ATTN_UNSUPPORTED: return "TT_ATTN_UNSUPPORTED";
    case TT_ATTN_LAUNCH_FAIL: return "TT_ATTN_LAUNCH_FAIL";
    case TT_ATTN_TIMEOUT: return "TT_ATTN_TIMEOUT";
  }
  return "TT_ATTN_UNKNOWN";
}

TT_ATTN_API const char* tt_attn_last_error(void) { return g_last_error.c_str(); }

TT_ATTN_API int tt_attn_layout_supported(const void* ptr, const int64_t* strides) {
  if (ptr == nullptr || strides == nullptr) return 0;
  return (aligned16(ptr) && strides_ok(strides)) ? 1 : 0;
}

TT_ATTN_API size_t tt_attn_forward_workspace_size(int64_t batch, int64_t heads, int64_t q_len,
                                                  int64_t kv_len) {
  if (batch <= 0 || heads <= 0 || q_len <= 0 || kv_len <= 0 || kv_len > INT32_MAX ||
      q_len > kv_len)
    return 0;
  if (batch > INT32_MAX / heads) return 0;
  if (q_len > 1) {
    // Prefill: partial records of split query blocks (causal, past_len = kv_len - q_len).
    const int64_t bh = batch * heads;
    return prefill_workspace_bytes(bh, q_len, prefill_plan(bh, q_len, kv_len, kv_len - q_len));
  }
  // Short and medium caches take the cluster kernel, which needs no workspace.
  if (use_direct_decode(batch * heads, kv_len)) return 0;
  const int64_t bh = batch * heads;
  const int chunk = decode_chunk(bh, kv_len);
  const int64_t n_chunks = (kv_len + chunk - 1) / chunk;
  // Decode: the work counter, then (with more than one chunk) the per-sequence arrival
  // counters and the FP32 partials.
  size_t bytes = tt::decode::kCounterBytes;
  if (n_chunks > 1)
    bytes += decode_arrival_bytes(bh) + static_cast<size_t>(bh) * static_cast<size_t>(n_chunks) *
                                            tt::decode::PARTIAL * sizeof(float);
  return bytes;
}

TT_ATTN_API int tt_attn_device_supported(void) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  int major = 0;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return 0;
  return major == 10 ? 1 : 0;
}

TT_ATTN_API tt_attn_status tt_attn_device_status(unsigned* flags, int clear) {
  if (flags == nullptr) return fail(TT_ATTN_BAD_ARG, "flags must not be NULL");
  cudaError_t e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaMemcpyFromSymbol(flags, tt::g_tt_status, sizeof(unsigned));
  if (e == cudaSuccess && clear) {
    const unsigned zero = 0;
    e = cudaMemcpyToSymbol(tt::g_tt_status, &zero, sizeof(unsigned));
  }
  if (e != cudaSuccess) return fail(TT_ATTN_LAUNCH_FAIL, std::string("status read: ") + cudaGetErrorString(e));
  if (*flags & tt::TT_ERR_TIMEOUT) return TT_ATTN_TIMEOUT;
  return (*flags & tt::TT_ERR_RANGE) ? TT_ATTN_BAD_ARG : TT_ATTN_OK;
}

TT_ATTN_API tt_attn_status tt_rope_append_bf16(
    const void* qkv, int64_t batch, int64_t q_len, int64_t heads, const float* cos,
    const float* sin, int64_t table_len, int64_t position, const int64_t* position_dev,
    void* q_out, void* cache_k, const int64_t* ck_strides, void* cache_v,
    const int64_t* cv_strides, int64_t capacity, void* stream) {
  if (!qkv || !cos || !sin || !q_out || !cache_k || !cache_v || !ck_strides || !cv_strides)
    return fail(TT_ATTN_BAD_ARG, "rope_append: pointers must not be NULL");
  if (batch <= 0 || q_len <= 0 || heads <= 0 || capacity <= 0 || table_len <= 0)
    return fail(TT_ATTN_BAD_ARG, "rope_append: sizes must be positive");
  if (ck_strides[3] != 1 || cv_strides[3] != 1)
    return fail(TT_ATTN_BAD_ARG, "rope_append: cache rows must be contiguous (last stride 1)");
  for (int i = 0; i < 3; ++i)
    if (ck_strides[i] % 2 != 0 || cv_strides[i] % 2 != 0)
      return fail(TT_ATTN_BAD_ARG, "rope_append: cache strides must be even (4-byte pairs)");
  for (const void* ptr : {qkv, static_cast<const void*>(q_out), static_cast<const void*>(cache_k),
                          static_cast<const void*>(cache_v), static_cast<const void*>(cos),
                          static_cast<const void*>(sin)})
    if (reinterpret_cast<uintptr_t>(ptr) % 4 != 0)
      return fail(TT_ATTN_BAD_ARG, "rope_append: pointers must be 4-byte aligned");
  const int64_t max_rows = static_cast<int64_t>(INT32_MAX) * tt::rope::ROWS_PER_BLOCK;
  if (batch > INT32_MAX || q_len > INT32_MAX || heads > INT32_MAX ||
      q_len > max_rows / heads / batch)
    return fail(TT_ATTN_BAD_ARG, "rope_append: shape exceeds the supported grid");
  const int64_t rows = batch * q_len * heads;
  if (position_dev == nullptr &&
      (position < 0 || position + q_len > capacity || position + q_len > table_len))
    return fail(TT_ATTN_BAD_ARG, "rope_append: position + q_len exceeds the cache capacity or "
                                 "the cos/sin table");
  int dev = 0;
  tt_attn_status st = prepare_device(&dev);
  if (st != TT_ATTN_OK) return st;
  tt::rope::Params p{};
  p.qkv = static_cast<const __nv_bfloat16*>(qkv);
  p.B = static_cast<int>(batch);
  p.T = static_cast<int>(q_len);
  p.H = static_cast<int>(heads);
  p.cos = cos;
  p.sin = sin;
  p.table_len = table_len;
  p.position = position;
  p.position_dev = reinterpret_cast<const long long*>(position_dev);
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.cache_k = static_cast<__nv_bfloat16*>(cache_k);
  p.cache_v = static_cast<__nv_bfloat16*>(cache_v);
  p.ck_s0 = ck_strides[0]; p.ck_s1 = ck_strides[1]; p.ck_s2 = ck_strides[2];
  p.cv_s0 = cv_strides[0]; p.cv_s1 = cv_strides[1]; p.cv_s2 = cv_strides[2];
  p.capacity = capacity;
  const unsigned grid =
      static_cast<unsigned>((rows + tt::rope::ROWS_PER_BLOCK - 1) / tt::rope::ROWS_PER_BLOCK);
  tt::rope::rope_append_kernel<<<grid, tt::rope::THREADS, 0, static_cast<cudaStream_t>(stream)>>>(p);
  return check_launch("rope_append_kernel launch");
}

TT_ATTN_API tt_attn_status tt_qkv_rope_append_bf16(
    const void* hidden, int64_t batch, int64_t q_len, int64_t dim, const void* w_qkv,
    int64_t heads, const float* cos, const float* sin, int64_t table_len, int64_t position,
    const int64_t* position_dev, void* q_out, void* cache_k, const int64_t* ck_strides,
    void* cache_v, const int64_t* cv_strides, int64_t capacity, void* stream) {
  namespace qr = tt::qkv_rope;
  if (!hidden || !w_qkv || !cos || !sin || !q_out || !cache_k || !cache_v || !ck_strides ||
      !cv_strides)
    return fail(TT_ATTN_BAD_ARG, "qkv_rope_append: pointers must not be NULL");
  if (batch <= 0 || q_len <= 0 || heads <= 0 || dim <= 0 || capacity <= 0 || table_len <= 0)
    return fail(TT_ATTN_BAD_ARG, "qkv_rope_append: sizes must be positive");
  if (dim % qr::BK != 0)
    return fail(TT_ATTN_UNSUPPORTED, "qkv_rope_append: the input dimension must be a multiple of 64");
  if (batch > INT32_MAX / q_len || heads > INT32_MAX / (3 * TT_ATTN_HEAD_DIM) ||
      dim > INT32_MAX)
    return fail(TT_ATTN_BAD_ARG, "qkv_rope_append: shape exceeds the supported grid");
  if (ck_strides[3] != 1 || cv_strides[3] != 1)
    return fail(TT_ATTN_BAD_ARG, "qkv_rope_append: cache rows must be contiguous (last stride 1)");
  for (int i = 0; i < 3; ++i)
    if (ck_strides[i] % 8 != 0 || cv_strides[i] % 8 != 0)
      return fail(TT_ATTN_BAD_ARG,
                  "qkv_rope_append: cache strides must be multiples of 8 elements (16-byte rows)");
  for (const void* ptr : {hidden, w_qkv, static_cast<const void*>(q_out),
                          static_cast<const void*>(cache_k), static_cast<const void*>(cache_v),
                          static_cast<const void*>(cos), static_cast<const void*>(sin)})
    if (!aligned16(ptr))
      return fail(TT_ATTN_BAD_ARG, "qkv_rope_append: pointers must be 16-byte aligned");
  if (position_dev == nullptr &&
      (position < 0 || position + q_len > capacity || position + q_len > table_len))
    return fail(TT_ATTN_BAD_ARG, "qkv_rope_append: position + q_len exceeds the cache capacity "
                                 "or the cos/sin table");
  const int64_t rows = batch * q_len;
  const int64_t n = 3 * heads * TT_ATTN_HEAD_DIM;
  const int64_t m_tiles = (rows + qr::BM - 1) / qr::BM;
  if (m_tiles > 65535) return fail(TT_ATTN_BAD_ARG, "qkv_rope_append: too many rows for the grid");
  int dev = 0, sm_count = 0;
  tt_attn_status st = prepare_device(&dev, &sm_count);
  if (st != TT_ATTN_OK) return st;
  const QkvRopePlan pl = qkv_rope_plan(rows, heads, dim, dev, sm_count);
  // One row tile: the h box covers only the rows that exist (TMA fills past M with zeros).
  const uint32_t box_rows = pl.splitk ? static_cast<uint32_t>(pl.red_rows)
                                      : static_cast<uint32_t>(qr::BM);
  CUtensorMap tm_h, tm_w;
  std::string err;
  if (!encode_map_2d(&tm_h, hidden, rows, dim, box_rows, &err) ||
      !encode_map_2d(&tm_w, w_qkv, n, dim, static_cast<uint32_t>(pl.bn), &err))
    return fail(TT_ATTN_UNSUPPORTED, err);
  qr::Params p{};
  p.M = static_cast<int>(rows);
  p.T = static_cast<int>(q_len);
  p.H = static_cast<int>(heads);
  p.K = static_cast<int>(dim);
  p.cos = cos;
  p.sin = sin;
  p.table_len = table_len;
  p.position = position;
  p.position_dev = reinterpret_cast<const long long*>(position_dev);
  p.q_out = static_cast<__nv_bfloat16*>(q_out);
  p.cache_k = static_cast<__nv_bfloat16*>(cache_k);
  p.cache_v = static_cast<__nv_bfloat16*>(cache_v);
  p.ck_s0 = ck_strides[0]; p.ck_s1 = ck_strides[1]; p.ck_s2 = ck_strides[2];
  p.cv_s0 = cv_strides[0]; p.cv_s1 = cv_strides[1]; p.cv_s2 = cv_strides[2];
  p.capacity = capacity;
  p.stage_tx_bytes = (box_rows + static_cast<uint32_t>(pl.bn)) * qr::BK * 2;
  p.n_tiles = static_cast<int>(pl.n_tiles);
  p.m_tiles = static_cast<int>(pl.m_tiles);
  p.red_rows = pl.red_rows;
  const cudaError_t le = launch_qkv_rope(pl, tm_h, tm_w, p, static_cast<cudaStream_t>(stream));
  if (le != cudaSuccess)
    return fail(TT_ATTN_LAUNCH_FAIL, std::string("qkv_rope_append launch: ") + cudaGetErrorString(le));
  return check_launch("qkv_rope_append launch");
}

// Backward workspace: -LSE * log2(e) and -D per query row, each [B, H, Tq_pad] FP32 with Tq
// padded to whole 128-row tiles (so every tile's rows are one aligned 512-byte copy), then the
// FP32 dQ accumulator [B, H, Tq, 64] that the fused kernel reduces into, then the persistent
// kernel's work counter (16 bytes, keeping the total a multiple of 16).
constexpr size_t kBackwardCounterBytes = 16;

// bwd_persistent_kernel is the default; TT_ATTN_BWD_PERSISTENT=0 in the environment (read once
// per process) selects the one-CTA-per-key-tile bwd_fused_kernel instead.
bool use_persistent_backward() {
  static const bool on = [] {
    const char* v = std::getenv("TT_ATTN_BWD_PERSISTENT");
    return !(v != nullptr && v[0] == '0' && v[1] == '\0');
  }();
  return on;
}

int64_t backward_q_pad(int64_t q_len) {
  const int64_t t = tt::backward::fused::T;
  return (q_len + t - 1) / t * t;
}

TT_ATTN_API size_t tt_attn_backward_workspace_size(int64_t batch, int64_t heads, int64_t q_len) {
  if (batch <= 0 || heads <= 0 || q_len <= 0 || batch > INT32_MAX / heads || q_len > INT32_MAX)
    return 0;
  const int64_t bh = batch * heads;
  return 2 * static_cast<size_t>(bh * backward_q_pad(q_len)) * sizeof(float) +
         static_cast<size_t>(bh * q_len) * TT_ATTN_HEAD_DIM * sizeof(float) +
         kBackwardCounterBytes;
}

}  // extern "C"

namespace {

// The deterministic backward: row sums D (first bh * Tq floats of the workspace), then the dQ
// kernel (128-row query tiles over 64-key steps) and the dK/dV kernel (128-key tiles over
// 64-row query steps); each output element is accumulated by one CTA in a fixed order.
tt_attn_status backward_deterministic(const void* q, const void* k, const void* v,
                                      const void* dout, const void* out, const float* lse,
                                      const Shape4& qs, const Shape4& ks, const Shape4& vs,
                                      const Shape4& dos, int64_t batch, int64_t heads,
                                      int64_t q_len, int64_t kv_len, int64_t past_len, void* dq,
                                      void* dk, void* dv, float* D, cudaStream_t cs) {
  namespace det = tt::backward_det;
  const int64_t bh = batch * heads;
  const int64_t rows = bh * q_len;
  const int64_t q_tiles = (q_len + det::TILE - 1) / det::TILE;
  const int64_t k_tiles = (kv_len + det::TILE - 1) / det::TILE;
  if (q_tiles > INT32_MAX / bh)
    return fail(TT_ATTN_BAD_ARG, "attention backward shape exceeds the supported CUDA grid limits");
  det::PreParams pp{};
  pp.rows = rows;
  pp.dO = static_cast<const __nv_bfloat16*>(dout);
  pp.O = static_cast<const __nv_bfloat16*>(out);
  pp.D = D;
  const int64_t pre_blocks = (rows + det::PRE_ROWS_PER_BLOCK - 1) / det::PRE_ROWS_PER_BLOCK;
  det::bwd_preprocess_kernel<<<static_cast<unsigned>(pre_blocks), 256, 0, cs>>>(pp);
  tt_attn_status st = check_launch("bwd_preprocess_kernel (deterministic) launch");
  if (st != TT_ATTN_OK) return st;
  // The dQ kernel reads Q / dO in 128-row tiles and K / V in 64-row steps; the dK/dV kernel
  // the other way round.
  constexpr unsigned tile = det::TILE, step = det::STEP;
  CUtensorMap tmq_t, tmdo_t, tmk_s, tmv_s, tmq_s, tmdo_s, tmk_t, tmv_t;
  std::string err;
  if (!encode_map(&tmq_t, q, qs, &err, tile) || !encode_map(&tmdo_t, dout, dos, &err, tile) ||
      !encode_map(&tmk_s, k, ks, &err, step) || !encode_map(&tmv_s, v, vs, &err, step) ||
      !encode_map(&tmq_s, q, qs, &err, step) || !encode_map(&tmdo_s, dout, dos, &err, step) ||
      !encode_map(&tmk_t, k, ks, &err, tile) || !encode_map(&tmv_t, v, vs, &err, tile))
    return fail(TT_ATTN_UNSUPPORTED, err);
  det::Params p{};
  p.B = static_cast<int>(batch);
  p.H = static_cast<int>(heads);
  p.Tq = static_cast<int>(q_len);
  p.Tk = static_cast<int>(kv_len);
  p.past_len = static_cast<int>(past_len);
  p.lse = lse;
  p.D = D;
  p.n_tiles = static_cast<int>(q_tiles);
  p.out0 = static_cast<__nv_bfloat16*>(dq);
  det::bwd_dq_kernel<<<static_cast<unsigned>(bh * q_tiles), det::THREADS, det::kSmemQ, cs>>>(
      tmq_t, tmk_s, tmv_s, tmdo_t, p);
  if ((st = check_launch("bwd_dq_kernel launch")) != TT_ATTN_OK) return st;
  p.n_tiles = static_cast<int>(k_tiles);
  p.out0 = static_cast<__nv_bfloat16*>(dk);
  p.out1 = static_cast<__nv_bfloat16*>(dv);
  det::bwd_dkdv_kernel<<<static_cast<unsigned>(bh * k_tiles), det::THREADS, det::kSmemKV, cs>>>(
      tmq_s, tmk_t, tmv_t, tmdo_s, p);
  return check_launch("bwd_dkdv_kernel launch");
}

// Both backward entry points: shared validation, then the fused path (dQ contributions of
// different key tiles added with reduce-adds in timing-dependent order) or the deterministic
// two-kernel path.
tt_attn_status backward_impl(
    bool deterministic, const void* q, const int64_t* q_strides, const void* k,
    const int64_t* k_strides, const void* v, const int64_t* v_strides, const void* dout,
    const void* out, const float* lse, int64_t batch, int64_t heads, int64_t q_len,
    int64_t kv_len, int64_t head_dim, int64_t past_len, void* dq, void* dk, void* dv,
    void* workspace, size_t workspace_bytes, void* stream) {
  // ---- validation: everything is checked before any CUDA call
  if (!q || !k || !v || !dout || !out || !lse || !dq || !dk || !dv || !q_strides || !k_strides ||
      !v_strides)
    return fail(TT_ATTN_BAD_ARG, "q, k, v, dO, O, LSE, dq, dk, dv and the stride arrays must not "
                                 "be NULL");
  if (head_dim != TT_ATTN_HEAD_DIM)
    return fail(TT_ATTN_BAD_ARG, "attention currently supports only head_dim=64");
  if (batch <= 0 || heads <= 0 || q_len <= 0 || kv_len <= 0)
    return fail(TT_ATTN_BAD_ARG, "attention batch, heads and sequence lengths must be positive");
  if (past_len < 0) return fail(TT_ATTN_BAD_ARG, "past_len must be non-negative");
  if (kv_len < q_len || past_len != kv_len - q_len)
    return fail(TT_ATTN_BAD_ARG, "expected Tk == past_len + Tq");
  if (q_len > INT32_MAX || kv_len > INT32_MAX)
    return fail(TT_ATTN_BAD_ARG, "bf16 attention sequence lengths must fit int32 (Tk <= INT32_MAX)");
  if (batch > INT32_MAX / heads)
    return fail(TT_ATTN_BAD_ARG, "attention backward shape exceeds the supported CUDA grid limits");
  const int64_t bh = batch * heads;
  const int64_t k_tiles = (kv_len + tt::backward::fused::T - 1) / tt::backward::fused::T;
  const int64_t q_pad = backward_q_pad(q_len);
  const int64_t rows = bh * q_len, pad_rows = bh * q_pad;
  // Query rows padded to whole tiles are int32 in the kernels; every grid must fit int32.
  if (q_pad > INT32_MAX || k_tiles > INT32_MAX / bh ||
      (pad_rows + tt::backward::PRE_ROWS_PER_BLOCK - 1) / tt::backward::PRE_ROWS_PER_BLOCK >
          INT32_MAX ||
      (rows * (TT_ATTN_HEAD_DIM / 8) + 255) / 256 > INT32_MAX)
    return fail(TT_ATTN_BAD_ARG, "attention backward shape exceeds the supported CUDA grid limits");
  const Shape4 qs = canonical(batch, heads, q_len, q_strides);
  const Shape4 ks = canonical(batch, heads, kv_len, k_strides);
  const Shape4 vs = canonical(batch, heads, kv_len, v_strides);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !strides_ok(qs.stride) ||
      !strides_ok(ks.stride) || !strides_ok(vs.stride))
    return fail(TT_ATTN_UNSUPPORTED,
                "q/k/v need a unit last stride, other strides in multiples of 8 elements and "
                "16-byte aligned bases; copy to aligned contiguous storage first");
  for (const void* ptr : {dout, out, static_cast<const void*>(dq), static_cast<const void*>(dk),
                          static_cast<const void*>(dv)})
    if (!aligned16(ptr))
      return fail(TT_ATTN_BAD_ARG, "dO, O, dq, dk and dv must be contiguous and 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(lse) % 4 != 0)
    return fail(TT_ATTN_BAD_ARG, "LSE must be 4-byte aligned");
  const size_t ws_needed = tt_attn_backward_workspace_size(batch, heads, q_len);
  if (workspace == nullptr || workspace_bytes < ws_needed || !aligned16(workspace))
    return fail(TT_ATTN_BAD_ARG, "workspace is smaller than tt_attn_backward_workspace_size() "
                                 "or not 16-byte aligned");

  int dev = 0, sm_count = 0;
  tt_attn_status st = prepare_device(&dev, &sm_count);
  if (st != TT_ATTN_OK) return st;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  const int64_t cstr[4] = {heads * q_len * TT_ATTN_HEAD_DIM, q_len * TT_ATTN_HEAD_DIM,
                           TT_ATTN_HEAD_DIM, 1};
  const Shape4 dos = canonical(batch, heads, q_len, cstr);
  if (deterministic)
    return backward_deterministic(q, k, v, dout, out, lse, qs, ks, vs, dos, batch, heads, q_len,
                                  kv_len, past_len, dq, dk, dv, static_cast<float*>(workspace), cs);
  float* nlse2 = static_cast<float*>(workspace);
  float* nd = nlse2 + pad_rows;
  float* dq_acc = nd + pad_rows;
  unsigned int* next_item = reinterpret_cast<unsigned int*>(dq_acc + rows * TT_ATTN_HEAD_DIM);

  constexpr unsigned tile = tt::backward::fused::T;
  CUtensorMap tmq, tmdo, tmk, tmv, tmacc;
  std::string err;
  if (!encode_map(&tmq, q, qs, &err, tile) || !encode_map(&tmdo, dout, dos, &err, tile) ||
      !encode_map(&tmk, k, ks, &err, tile) || !encode_map(&tmv, v, vs, &err, tile) ||
      !encode_map_f32(&tmacc, dq_acc, dos, &err, tt::backward::fused::DQ_BOX_ROWS))
    return fail(TT_ATTN_UNSUPPORTED, err);

  tt::backward::PreParams pp{};
  pp.rows = pad_rows;
  pp.Tq = static_cast<int>(q_len);
  pp.Tq_pad = static_cast<int>(q_pad);
  pp.dO = static_cast<const __nv_bfloat16*>(dout);
  pp.O = static_cast<const __nv_bfloat16*>(out);
  pp.lse = lse;
  pp.nlse2 = nlse2;
  pp.nd = nd;
  pp.dq_acc = dq_acc;
  pp.next_item = next_item;
  const int64_t pre_blocks =
      (pad_rows + tt::backward::PRE_ROWS_PER_BLOCK - 1) / tt::backward::PRE_ROWS_PER_BLOCK;
  tt::backward::bwd_preprocess_kernel<<<static_cast<unsigned>(pre_blocks), 256, 0, cs>>>(pp);
  if ((st = check_launch("bwd_preprocess_kernel launch")) != TT_ATTN_OK) return st;

  if (use_persistent_backward()) {
    tt::backward::persist::Params pq{};
    pq.B = static_cast<int>(batch);
    pq.H = static_cast<int>(heads);
    pq.Tq = static_cast<int>(q_len);
    pq.Tk = static_cast<int>(kv_len);
    pq.past_len = static_cast<int>(past_len);
    pq.n_k_tiles = static_cast<int>(k_tiles);
    pq.Tq_pad = static_cast<int>(q_pad);
    pq.n_items = static_cast<int>(bh * k_tiles);
    pq.nlse2 = nlse2;
    pq.nd = nd;
    pq.dk = static_cast<__nv_bfloat16*>(dk);
    pq.dv = static_cast<__nv_bfloat16*>(dv);
    pq.next_item = next_item;
    const int64_t grid = std::min<int64_t>(bh * k_tiles, sm_count > 0 ? sm_count : 148);
    const cudaError_t ae = cudaFuncSetAttribute(tt::backward::persist::bwd_persistent_kernel,
                                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                static_cast<int>(tt::backward::persist::kSmemBytes));
    if (ae != cudaSuccess)
      return fail(TT_ATTN_LAUNCH_FAIL,
                  std::string("cudaFuncSetAttribute: ") + cudaGetErrorString(ae));
    tt::backward::persist::bwd_persistent_kernel<<<static_cast<unsigned>(grid),
                                                   tt::backward::persist::THREADS,
                                                   tt::backward::persist::kSmemBytes, cs>>>(
        tmq, tmk, tmv, tmdo, tmacc, pq);
    if ((st = check_launch("bwd_persistent_kernel launch")) != TT_ATTN_OK) return st;
  } else {
  tt::backward::fused::Params p{};
  p.B = static_cast<int>(batch);
  p.H = static_cast<int>(heads);
  p.Tq = static_cast<int>(q_len);
  p.Tk = static_cast<int>(kv_len);
  p.past_len = static_cast<int>(past_len);
  p.n_k_tiles = static_cast<int>(k_tiles);
  p.Tq_pad = static_cast<int>(q_pad);
  p.nlse2 = nlse2;
  p.nd = nd;
  p.dk = static_cast<__nv_bfloat16*>(dk);
  p.dv = static_cast<__nv_bfloat16*>(dv);
  tt::backward::fused::bwd_fused_kernel<<<static_cast<unsigned>(bh * k_tiles),
                                          tt::backward::fused::THREADS,
                                          tt::backward::fused::kSmemBytes, cs>>>(
      tmq, tmk, tmv, tmdo, tmacc, p);
  if ((st = check_launch("bwd_fused_kernel launch")) != TT_ATTN_OK) return st;
  }

  tt::backward::fused::ConvertParams cp{};
  cp.rows = rows;
  cp.acc = dq_acc;
  cp.dq = static_cast<__nv_bfloat16*>(dq);
  const int64_t conv_blocks = (rows * (TT_ATTN_HEAD_DIM / 8) + 255) / 256;
  tt::backward::fused::bwd_dq_convert_kernel<<<static_cast<unsigned>(conv_blocks), 256, 0, cs>>>(cp);
  return check_launch("bwd_dq_convert_kernel launch");
}

}  // namespace

extern "C" {

TT_ATTN_API tt_attn_status tt_attn_backward_bf16(
    const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides, const void* dout, const void* out, const float* lse,
    int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int64_t head_dim,
    int64_t past_len, void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
    void* stream) {
  return backward_impl(false, q, q_strides, k, k_strides, v, v_strides, dout, out, lse, batch,
                       heads, q_len, kv_len, head_dim, past_len, dq, dk, dv, workspace,
                       workspace_bytes, stream);
}

TT_ATTN_API tt_attn_status tt_attn_backward_bf16_deterministic(
    const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides, const void* dout, const void* out, const float* lse,
    int64_t batch, int64_t heads, int64_t q_len, int64_t kv_len, int64_t head_dim,
    int64_t past_len, void* dq, void* dk, void* dv, void* workspace, size_t workspace_bytes,
    void* stream) {
  return backward_impl(true, q, q_strides, k, k_strides, v, v_strides, dout, out, lse, batch,
                       heads, q_len, kv_len, head_dim, past_len, dq, dk, dv, workspace,
                       workspace_bytes, stream);
}

TT_ATTN_API tt_attn_status tt_attn_selftest_wait_timeout(int64_t budget_cycles, void* stream) {
  if (budget_cycles < 1 || budget_cycles > tt::selftest::kMaxSelftestBudget)
    return fail(TT_ATTN_BAD_ARG, "budget_cycles must be in [1, 1e9]");
  int dev = 0;
  tt_attn_status st = prepare_device(&dev);
  if (st != TT_ATTN_OK) return st;
  tt::selftest::wait_timeout_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<long long>(budget_cycles));
  return check_launch("wait_timeout_kernel launch");
}

TT_ATTN_API tt_attn_status tt_attn_forward_bf16(
    const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides, int64_t batch, int64_t heads, int64_t q_len,
    int64_t kv_len, int64_t head_dim, int64_t past_len, const int32_t* kv_lens, void* out,
    float* lse, void* workspace, size_t workspace_bytes, void* stream) {
  // ---- validation: everything is checked before any CUDA call
  if (!q || !k || !v || !out || !lse || !q_strides || !k_strides || !v_strides)
    return fail(TT_ATTN_BAD_ARG, "q, k, v, out, lse and the stride arrays must not be NULL");
  if (head_dim != TT_ATTN_HEAD_DIM)
    return fail(TT_ATTN_BAD_ARG, "attention currently supports only head_dim=64");
  if (batch <= 0 || heads <= 0 || q_len <= 0 || kv_len <= 0)
    return fail(TT_ATTN_BAD_ARG, "attention batch, heads and sequence lengths must be positive");
  if (past_len < 0) return fail(TT_ATTN_BAD_ARG, "past_len must be non-negative");
  if (kv_len < q_len || past_len != kv_len - q_len)
    return fail(TT_ATTN_BAD_ARG, "expected Tk == past_len + Tq");
  if (q_len > INT32_MAX || kv_len > INT32_MAX)
    return fail(TT_ATTN_BAD_ARG, "bf16 attention sequence lengths must fit int32 (Tk <= INT32_MAX)");
  if (kv_lens != nullptr && q_len != 1)
    return fail(TT_ATTN_BAD_ARG, "kv_lens requires single-token decode (Tq == 1)");
  if (batch > INT32_MAX / heads)
    return fail(TT_ATTN_BAD_ARG, "attention shape exceeds the supported CUDA grid limits");
  const int64_t bh = batch * heads;
  const bool is_decode = (q_len == 1);
  int64_t grid = 0;
  int chunk = 0;
  int64_t n_chunks = 0;
  if (is_decode) {
    chunk = decode_chunk(bh, kv_len);
    n_chunks = (kv_len + chunk - 1) / chunk;
    if (n_chunks > INT32_MAX / bh)
      return fail(TT_ATTN_BAD_ARG, "attention shape exceeds the supported CUDA grid limits");
    grid = bh * n_chunks;  // work items; the persistent grid is sized below
  } else {
    const int64_t n_qblocks = (q_len + tt::prefill::BLOCK_M - 1) / tt::prefill::BLOCK_M;
    if (n_qblocks > INT32_MAX / bh)
      return fail(TT_ATTN_BAD_ARG, "attention shape exceeds the supported CUDA grid limits");
    grid = bh * n_qblocks;  // without a KV split; with one, at most 2 x 148 + the parts
  }

  const Shape4 qs = canonical(batch, heads, q_len, q_strides);
  const Shape4 ks = canonical(batch, heads, kv_len, k_strides);
  const Shape4 vs = canonical(batch, heads, kv_len, v_strides);
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !strides_ok(qs.stride) ||
      !strides_ok(ks.stride) || !strides_ok(vs.stride))
    return fail(TT_ATTN_UNSUPPORTED,
                "q/k/v need a unit last stride, other strides in multiples of 8 elements and "
                "16-byte aligned bases; copy to aligned contiguous storage first");
  if (!aligned16(out)) return fail(TT_ATTN_BAD_ARG, "out must be 16-byte aligned");
  const size_t ws_needed = tt_attn_forward_workspace_size(batch, heads, q_len, kv_len);
  if (ws_needed > 0 && (workspace == nullptr || workspace_bytes < ws_needed))
    return fail(TT_ATTN_BAD_ARG, "workspace is smaller than tt_attn_forward_workspace_size()");

  int dev = 0, sm_count = 0;
  tt_attn_status st = prepare_device(&dev, &sm_count);
  if (st != TT_ATTN_OK) return st;
  cudaStream_t cs = reinterpret_cast<cudaStream_t>(stream);

  if (is_decode && use_direct_decode(bh, kv_len)) {
    // One cluster of `splits` CTAs per (batch, head); no workspace, one launch.
    namespace dd = tt::decode_direct;
    tt::decode_direct::Params p{};
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.k = static_cast<const __nv_bfloat16*>(k);
    p.v = static_cast<const __nv_bfloat16*>(v);
    p.q_sb = qs.stride[0];
    p.q_sh = qs.stride[1];
    p.k_sb = ks.stride[0];
    p.k_sh = ks.stride[1];
    p.k_st = ks.stride[2];
    p.v_sb = vs.stride[0];
    p.v_sh = vs.stride[1];
    p.v_st = vs.stride[2];
    p.kv_lens = kv_lens;
    p.B = static_cast<int>(batch);
    p.H = static_cast<int>(heads);
    p.Tk = static_cast<int>(kv_len);
    const int64_t passes_total = (kv_len + dd::KEYS_PER_PASS - 1) / dd::KEYS_PER_PASS;
    // CTAs per sequence: enough to fill three CTAs per SM, at most 4 (and one per chunk).
    // Measured on B200 (graph replay, H = 12): B * H = 12 / 96 best at 4, 192 at 2, 384 and
    // 768 at 1 (e.g. B = 32, Tk = 1024: 24.3 us at 1 against 39.5 at 8; B = 8, Tk = 4096:
    // 23.9 at 4 against 30.3 at 8): with a two-stage ring per CTA, fewer and longer CTAs
    // stream their chunks back to back, while each extra CTA pays the launch, the first load's
    // latency and the cluster merge.
    p.splits = static_cast<int>(std::max<int64_t>(
        1, std::min<int64_t>({kDirectDecodeMaxSplits, passes_total,
                              (3 * static_cast<int64_t>(sm_count > 0 ? sm_count : 148)) / bh})));
    p.keys_per_cta =
        static_cast<int>((passes_total + p.splits - 1) / p.splits) * dd::KEYS_PER_PASS;
    p.o = static_cast<__nv_bfloat16*>(out);
    p.lse = lse;
    p.scale_log2 = kScaleLog2;
    CUtensorMap tmk, tmv;
    std::string err;
    if (!encode_map(&tmk, k, ks, &err, dd::KEYS_PER_PASS) ||
        !encode_map(&tmv, v, vs, &err, dd::KEYS_PER_PASS))
      return fail(TT_ATTN_UNSUPPORTED, err);
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(static_cast<unsigned>(bh * p.splits), 1, 1);
    cfg.blockDim = dim3(dd::THREADS, 1, 1);
    cfg.dynamicSmemBytes = dd::kSmemBytes;
    cfg.stream = cs;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(p.splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t le = cudaLaunchKernelEx(&cfg, dd::decode_direct_kernel, tmk, tmv, p);
    if (le != cudaSuccess)
      return fail(TT_ATTN_LAUNCH_FAIL,
                  std::string("decode_direct_kernel launch: ") + cudaGetErrorString(le));
    return check_launch("decode_direct_kernel launch");
  }
  if (is_decode) {
    tt::decode::Params p{};
    p.q = static_cast<const __nv_bfloat16*>(q);
    p.k = static_cast<const __nv_bfloat16*>(k);
    p.v = static_cast<const __nv_bfloat16*>(v);
    p.q_sb = qs.stride[0];
    p.q_sh = qs.stride[1];
    p.k_sb = ks.stride[0];
    p.k_sh = ks.stride[1];
    p.k_st = ks.stride[2];
    p.v_sb = vs.stride[0];
    p.v_sh = vs.stride[1];
    p.v_st = vs.stride[2];
    p.kv_lens = kv_lens;
    p.B = static_cast<int>(batch);
    p.H = static_cast<int>(heads);
    p.Tk = static_cast<int>(kv_len);
    p.chunk = chunk;
    p.n_chunks = static_cast<int>(n_chunks);
    p.o = static_cast<__nv_bfloat16*>(out);
    p.lse = lse;
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    const size_t arrival_bytes = n_chunks > 1 ? decode_arrival_bytes(bh) : 0;
    p.counter = reinterpret_cast<unsigned*>(ws);
    p.arrivals = reinterpret_cast<unsigned*>(ws + tt::decode::kCounterBytes);
    p.partials = reinterpret_cast<float*>(ws + tt::decode::kCounterBytes + arrival_bytes);
    p.scale_log2 = kScaleLog2;
    // The CTAs take work items from a counter, and count each split sequence's published
    // partials, from zero: one memset clears both.
    const size_t clear =
        n_chunks > 1 ? tt::decode::kCounterBytes + arrival_bytes : sizeof(unsigned);
    const cudaError_t me = cudaMemsetAsync(ws, 0, clear, cs);
    if (me != cudaSuccess)
      return fail(TT_ATTN_LAUNCH_FAIL, std::string("cudaMemsetAsync(decode counters): ") +
                                           cudaGetErrorString(me));
    // Persistent grid: one CTA per SM streams work items; no more CTAs than items.
    const int64_t ctas = std::min<int64_t>(sm_count, grid);
    tt::decode::decode_split_kernel<<<static_cast<unsigned>(ctas), tt::decode::THREADS,
                                      tt::decode::kSmemBytes, cs>>>(p);
    return check_launch("decode_split_kernel launch");
  }

  CUtensorMap tmq, tmk, tmv;
  std::string err;
  constexpr unsigned kv_box = tt::prefill::BN;
  if (!encode_map(&tmq, q, qs, &err) || !encode_map(&tmk, k, ks, &err, kv_box) ||
      !encode_map(&tmv, v, vs, &err, kv_box))
    return fail(TT_ATTN_UNSUPPORTED, err);
  const PrefillPlan plan = prefill_plan(bh, q_len, kv_len, past_len);
  tt::prefill::Params p{};
  p.B = static_cast<int>(batch);
  p.H = static_cast<int>(heads);
  p.Tq = static_cast<int>(q_len);
  p.Tk = static_cast<int>(kv_len);
  p.past_len = static_cast<int>(past_len);
  p.n_qblocks = static_cast<int>((q_len + tt::prefill::BLOCK_M - 1) / tt::prefill::BLOCK_M);
  p.o = static_cast<__nv_bfloat16*>(out);
  p.lse = lse;
  p.scale_log2 = kScaleLog2;
  p.part_tiles = plan.part_tiles;
  p.max_parts = plan.max_parts;
  p.first_split_qb = plan.first_split_qb;
  p.partials = static_cast<float*>(workspace);
  if (plan.part_tiles == 0) {
    tt::prefill::attention_prefill_kernel<false>
        <<<static_cast<unsigned>(plan.ctas), tt::prefill::THREADS, tt::prefill::kSmemBytes, cs>>>(
            tmq, tmk, tmv, p);
    return check_launch("attention_prefill_kernel launch");
  }
  tt::prefill::attention_prefill_kernel<true>
      <<<static_cast<unsigned>(plan.ctas), tt::prefill::THREADS, tt::prefill::kSmemBytes, cs>>>(
          tmq, tmk, tmv, p);
  if ((st = check_launch("attention_prefill_kernel launch")) != TT_ATTN_OK) return st;
  const int64_t rows = bh * (p.n_qblocks - plan.first_split_qb) * tt::prefill::BLOCK_M;
  const int64_t blocks = (rows + tt::prefill::COMBINE_WARPS - 1) / tt::prefill::COMBINE_WARPS;
  tt::prefill::prefill_combine_kernel<<<static_cast<unsigned>(blocks),
                                        tt::prefill::COMBINE_WARPS * 32, 0, cs>>>(p);
  return check_launch("prefill_combine_kernel launch");
}

}  // extern "C"

// ------------------------------------------------------------------ no-allocation decode
// Some callers cannot allocate device memory at the moment they decode: an inference server
// that reserved all of the GPU's memory for its own pools up front, a host language runtime
// (Go, Java, Rust) driving this library over its C ABI without a CUDA allocator of its own,
// or a latency-critical loop that must not enter the driver's allocator. For them the split-KV
// partials live in this file-scope device array instead of a caller-provided workspace.
// Every GPU that loads this library holds the array until the process exits.
namespace {
constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB of decode partials
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

// Host code must not use the array's name as a device address: it is a host-side stand-in.
// The device address is fetched with the device current, and fetched again whenever the
// thread's current context on that device is a different one (after cudaDeviceReset, or when
// the caller made a context of its own current), since the array lives once per context.
struct NoAllocScratch {
  void* ctx = nullptr;  // CUcontext the address belongs to
  void* ptr = nullptr;
};
NoAllocScratch g_noalloc_scratch_ptr[kMaxDevices];
std::mutex g_noalloc_mu;

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<CtxGetCurrentFn>(ptr);
  });
  return fn;
}
}  // namespace

extern "C" {

TT_ATTN_API tt_attn_status tt_attn_decode_bf16_noalloc(
    const void* q, const int64_t* q_strides, const void* k, const int64_t* k_strides,
    const void* v, const int64_t* v_strides, int64_t batch, int64_t heads, int64_t kv_len,
    const int32_t* kv_lens, void* out, float* lse, void* stream) {
  if (batch <= 0 || heads <= 0 || kv_len <= 0)
    return fail(TT_ATTN_BAD_ARG, "attention batch, heads and sequence lengths must be positive");
  const size_t need = tt_attn_forward_workspace_size(batch, heads, 1, kv_len);
  if (need > kNoAllocScratchBytes) {
    char buf[200];
    std::snprintf(buf, sizeof(buf),
                  "decode of this shape needs %zu bytes of scratch; the no-allocation entry point "
                  "holds at most %zu bytes: use tt_attn_forward_bf16 with a workspace",
                  need, kNoAllocScratchBytes);
    return fail(TT_ATTN_BAD_ARG, buf);
  }
  // The device check first: on a device without an sm_100 image the symbol lookup below would
  // fail with a less useful message than the forward entry point's UNSUPPORTED.
  int dev = 0;
  tt_attn_status st = prepare_device(&dev);
  if (st != TT_ATTN_OK) return st;
  CUcontext ctx = nullptr;
  CtxGetCurrentFn get_ctx = ctx_get_current_fn();
  if (get_ctx == nullptr || get_ctx(&ctx) != CUDA_SUCCESS || ctx == nullptr)
    return fail(TT_ATTN_LAUNCH_FAIL, "no current CUDA context for the no-allocation scratch");
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    NoAllocScratch& slot = g_noalloc_scratch_ptr[dev];
    if (slot.ptr == nullptr || slot.ctx != static_cast<void*>(ctx)) {
      void* ptr = nullptr;
      const cudaError_t se = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
      if (se != cudaSuccess || ptr == nullptr)
        return fail(TT_ATTN_LAUNCH_FAIL,
                    std::string("cudaGetSymbolAddress(no-allocation scratch): ") +
                        cudaGetErrorString(se));
      slot.ptr = ptr;
      slot.ctx = static_cast<void*>(ctx);
    }
    scratch = slot.ptr;
  }
  // Each call clears the counters it uses and writes every partial before it is read, so the
  // scratch needs no clearing between calls.
  return tt_attn_forward_bf16(q, q_strides, k, k_strides, v, v_strides, batch, heads, 1, kv_len,
                              TT_ATTN_HEAD_DIM, kv_len - 1, kv_lens, out, lse, scratch,
                              kNoAllocScratchBytes, stream);
}

}  // extern "C"
