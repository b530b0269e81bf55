// Paged GQA decode attention over a shared page pool, with split-KV and a log-sum-exp merge.
//
// Work decomposition, tensor-core path. The 16-token tiles of every (request, KV head) "segment"
// form one stream; each of the W resident warps owns an equal contiguous slice of it (stream-K),
// derived in-kernel from seq_lens, so the load is balanced whatever the context lengths. A segment
// cut between warps becomes "pieces": each piece writes its unnormalised partial (running max m,
// sum l, accumulator) to the workspace and a second small kernel merges them. Nothing waits on
// another warp.
//
// Work decomposition, generic path. A one-CTA plan kernel splits every request into units of
// consecutive pages per KV head; persistent CTAs take units from an atomic counter; the split whose
// counter increment completes a (request, KV head) merges its partials and resets the counter.
//
// Tensor-core path (fp16/bf16, head_dim 64/128/256, block_size % 16 == 0, <= 8 query heads per KV
// head). One warp streams 16-token tiles of K and V of its unit through a ring of shared-memory
// stages filled by 2-D TMA loads (128-byte swizzle, L2 evict-first, completion on one mbarrier per
// stage). Per tile:
//   S^T (16 tokens x 8 heads) = K_tile (16 x D) . Q^T (D x 8)      -- mma.m16n8k16, tokens on M
//   online softmax over the 16 tokens per head (max by 3 xor-shuffles, exp2 on the SFU)
//   O^T (D x 8 heads) += V_tile^T (D x 16) . P^T (16 x 8)          -- P^T moved to the B fragment
//                                                                    with movmatrix, V by ldmatrix.trans
// Putting tokens (not the 8 query heads) on the M=16 side fills every MMA with useful work. The
// contraction index of Q.K is permuted so that each thread reads K with conflict-free 16-byte
// shared loads (Q uses the same permutation, so the dot products are unchanged).
//
// Generic path (fp32 and every other shape): CUDA cores, one CTA per unit, warps interleave the
// tokens, warp-shuffle dot products and online softmax per query head, CTA merge through shared
// memory. Both paths accumulate in fp32; softmax probabilities are rounded to the KV dtype before
// the P.V product on the tensor-core path, as the reference does (src/reference_ops.py:357).
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>
#include <type_traits>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int kTargetUnits = 2048;   // the automatic split size aims at about this many units
constexpr int kMinSplitTokens = 128;  // ... but never splits below this many tokens
constexpr int kTcWarps = 4;           // warps per CTA of the tensor-core kernel
constexpr int kGenThreads = 128;      // threads per CTA of the generic kernel
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // bounded mbarrier waits: 2 s

struct WsHeader {
  int32_t num_units;        // generic path: units in the work list
  int32_t unit_counter;     // generic path: next unit to take
  int32_t pages_per_split;  // generic path: split size chosen by the plan
  int32_t reserved[61];
};
static_assert(sizeof(WsHeader) == 256, "header is one 256-byte line");

constexpr int kMaxStreamWarps = 1280;  // upper bound of tensor-core warps a launch may use (>= 148 SMs x 8)

struct WsLayout {
  int64_t counters_off, units_off, ml_off, acc_off, total;
  int64_t max_units, max_slots;
};

int64_t pages_per_split_min(int64_t block_size) {
  return std::max<int64_t>(1, kMinSplitTokens / block_size);
}

// One layout serves both paths: the generic path's unit list, per-(request, KV head) merge counters
// and partial results sized for the larger of the generic path's units and the tensor-core path's
// two partial slots per warp.
WsLayout ws_layout(int64_t batch, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim, int64_t max_blocks,
                   int64_t block_size, int64_t pages_per_split) {
  WsLayout w{};
  const int64_t group = num_kv_heads > 0 ? num_q_heads / num_kv_heads : 0;
  const int64_t bh = batch * num_kv_heads;
  if (pages_per_split > 0) {
    w.max_units = bh * ceil_div(std::max<int64_t>(max_blocks, 1), pages_per_split);
  } else {
    const int64_t by_table = bh * ceil_div(std::max<int64_t>(max_blocks, 1), pages_per_split_min(block_size));
    w.max_units = std::min<int64_t>(by_table, kTargetUnits + bh);
  }
  w.max_slots = std::max<int64_t>(w.max_units, 2 * kMaxStreamWarps);
  w.counters_off = 256;
  w.units_off = align_up(w.counters_off + bh * 4, 256);
  w.ml_off = align_up(w.units_off + w.max_units * 16, 256);
  w.acc_off = align_up(w.ml_off + w.max_slots * group * 8, 256);
  w.total = align_up(w.acc_off + w.max_slots * group * head_dim * 4, 256);
  return w;
}

struct Workspace {
  WsHeader* hdr;
  int32_t* counters;  // per (request, KV head): pieces finished; zero between calls
  int4* units;        // generic path: {request, (split << 8) | kv head, first page, end page}
  float2* part_ml;
  float* part_acc;
  int32_t max_units;
};

// ---- plan --------------------------------------------------------------------------------------------
template <typename I>
struct PlanArgs {
  const I* seq_lens;
  int64_t uniform_len;  // >= 0: every request has this length and seq_lens is ignored
  int32_t batch, num_kv_heads, num_q_heads;
  int32_t block_size;
  int32_t max_blocks;
  int32_t pages_per_split;  // <= 0: automatic
  int32_t pps_min;
  Workspace ws;
  char* out;  // rows of requests with L <= 0 are zeroed here
  int64_t o_sb, o_sh;  // bytes
  int32_t row_bytes;
  int32_t* error_flag;
};

template <typename I>
__device__ __forceinline__ int64_t request_len(const I* seq_lens, int64_t uniform_len, int64_t b) {
  return uniform_len >= 0 ? uniform_len : load_index(seq_lens, b);
}

template <typename I>
__global__ void __launch_bounds__(1024) decode_plan_kernel(PlanArgs<I> p) {
  __shared__ int64_t s_red[32];
  __shared__ int32_t s_scan[32];
  __shared__ int32_t s_pps;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nwarps = blockDim.x >> 5;
  auto pages_of = [&](int64_t b) -> int32_t {
    const int64_t len = request_len(p.seq_lens, p.uniform_len, b);
    if (len <= 0) return 0;
    int64_t np = (len + p.block_size - 1) / p.block_size;
    if (np > p.max_blocks) np = p.max_blocks;
    return static_cast<int32_t>(np);
  };
  // pass 1: total pages (for the automatic split size), flags, zero outputs of empty rows
  int64_t local = 0;
  for (int64_t b = tid; b < p.batch; b += blockDim.x) {
    const int64_t len = request_len(p.seq_lens, p.uniform_len, b);
    if (len > static_cast<int64_t>(p.max_blocks) * p.block_size) raise_device_error(p.error_flag, PKV_DEVERR_TABLE_TOO_SHORT);
    local += pages_of(b);
    if (len <= 0 && p.out != nullptr) {
      for (int h = 0; h < p.num_q_heads; ++h) {
        char* row = p.out + b * p.o_sb + h * p.o_sh;
        for (int i = 0; i < p.row_bytes; i += 2) *reinterpret_cast<uint16_t*>(row + i) = 0;
      }
    }
  }
  for (int off = 16; off > 0; off >>= 1) local += __shfl_xor_sync(0xffffffffu, local, off);
  if (lane == 0) s_red[warp] = local;
  __syncthreads();
  if (tid == 0) {
    int64_t total = 0;
    for (int w = 0; w < nwarps; ++w) total += s_red[w];
    int64_t pps = p.pages_per_split;
    if (pps <= 0) {
      pps = (total * p.num_kv_heads + kTargetUnits - 1) / kTargetUnits;
      if (pps < p.pps_min) pps = p.pps_min;
    }
    s_pps = static_cast<int32_t>(pps);
    p.ws.hdr->pages_per_split = s_pps;
    p.ws.hdr->unit_counter = 0;
  }
  for (int64_t i = tid; i < static_cast<int64_t>(p.batch) * p.num_kv_heads; i += blockDim.x) p.ws.counters[i] = 0;
  __syncthreads();
  const int32_t pps = s_pps;
  // pass 2: exclusive scan of units per request, in chunks of blockDim.x requests
  int32_t running = 0;
  for (int64_t chunk = 0; chunk < p.batch; chunk += blockDim.x) {
    const int64_t b = chunk + tid;
    const int32_t np = b < p.batch ? pages_of(b) : 0;
    const int32_t ns = (np + pps - 1) / pps;
    const int32_t n = ns * p.num_kv_heads;
    int32_t incl = n;
    for (int off = 1; off < 32; off <<= 1) {
      const int32_t v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    if (lane == 31) s_scan[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int32_t v = lane < nwarps ? s_scan[lane] : 0;
      for (int off = 1; off < 32; off <<= 1) {
        const int32_t t = __shfl_up_sync(0xffffffffu, v, off);
        if (lane >= off) v += t;
      }
      if (lane < nwarps) s_scan[lane] = v;
    }
    __syncthreads();
    const int32_t warp_base = warp > 0 ? s_scan[warp - 1] : 0;
    int32_t u = running + warp_base + incl - n;
    for (int32_t kvh = 0; kvh < p.num_kv_heads; ++kvh) {
      for (int32_t s = 0; s < ns; ++s, ++u) {
        if (u < p.ws.max_units) {
          p.ws.units[u] = make_int4(static_cast<int32_t>(b), (s << 8) | kvh, s * pps, min(np, (s + 1) * pps));
        }
      }
    }
    running += s_scan[nwarps - 1];
    __syncthreads();
  }
  if (tid == 0) {
    if (running > p.ws.max_units) {
      raise_device_error(p.error_flag, PKV_DEVERR_TABLE_TOO_SHORT);
      running = p.ws.max_units;
    }
    p.ws.hdr->num_units = running;
  }
}

// ---- tile stream (tensor-core path) ---------------------------------------------------------------------
// The 16-token tiles of all (request, KV head) segments form one stream of T tiles; warp w of W owns
// tiles [floor(w T / W), floor((w+1) T / W)). With W <= T every warp owns at least one tile, and the
// warps touching segment [a, e) are warp_of_tile(a) .. warp_of_tile(e - 1): that many "pieces" merge.
__device__ __forceinline__ int64_t warp_of_tile(int64_t t, int64_t total, int64_t warps) {
  return ((t + 1) * warps - 1) / total;
}

// ---- merge of split partials (one warp) ----------------------------------------------------------------
template <typename T>
__device__ void merge_splits_warp(const Workspace& ws, int first_unit, int ns, int group, int head_dim, T* out,
                                  int64_t o_sb, int64_t o_sh, int b, int q_head0, int lane) {
  for (int h = 0; h < group; ++h) {
    float mx = kNegInf;
    for (int s = lane; s < ns; s += 32) mx = fmaxf(mx, __ldcg(&ws.part_ml[(first_unit + s) * group + h]).x);
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float base = mx == kNegInf ? 0.f : mx;
    float lsum = 0.f;
    for (int s = lane; s < ns; s += 32) {
      const float2 ml = __ldcg(&ws.part_ml[(first_unit + s) * group + h]);
      lsum += ml.y * fast_exp2(ml.x - base);
    }
    for (int off = 16; off > 0; off >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
    T* orow = out + b * o_sb + (q_head0 + h) * o_sh;
    for (int d = lane; d < head_dim; d += 32) {
      float o = 0.f;
      for (int s = 0; s < ns; ++s) {
        const float2 ml = __ldcg(&ws.part_ml[(first_unit + s) * group + h]);
        const float w = fast_exp2(ml.x - base);
        o += w * __ldcg(&ws.part_acc[(static_cast<int64_t>(first_unit + s) * group + h) * head_dim + d]);
      }
      orow[d] = Elem<T>::from_f(o * inv);
    }
  }
}

// ---- tensor-core kernel -----------------------------------------------------------------------------------
template <typename I>
struct TcArgs {
  const void* q;
  int64_t q_sb, q_sh;  // elements
  const I* tables;
  int64_t table_stride;
  int32_t max_blocks;
  const I* seq_lens;
  int32_t num_pages, block_size;
  int32_t rows_per_page, rows_per_head;  // pool rows (of head_dim elements) per page / per KV head
  int32_t num_kv_heads, group;
  int32_t batch;
  int32_t pages_per_split;  // > 0: about this many pages per warp (fewer warps)
  float scale_log2;
  Workspace ws;
  void* out;
  int64_t o_sb, o_sh;  // elements
  int32_t* error_flag;
  // FP8 pools only: per-(slot, KV head) dequantisation scales, (pages, kv heads, block_size) strides
  const float* k_scales;
  const float* v_scales;
  int64_t scale_sp, scale_sh;  // floats
  int32_t chained;             // host side: launch with programmatic stream serialisation
  int32_t prefetch;            // start the page loads before waiting for the previous kernel
};

// F8: K/V pools hold e4m3 bytes. A stage then holds the fp8 K and V tiles (16 * D bytes each, 128-byte
// swizzled boxes of 128 elements); after the stages come the stages' 16 + 16 fp32 scales. Every TMA
// destination stays on a 1024-byte boundary (the 128-byte swizzle pattern the reads assume).
template <int D, bool F8 = false>
struct TcConfig {
  // fp8 tiles are half the bytes but cost more instructions (widening): twice the warps per CTA, each
  // with half the shared memory, keeps the bytes in flight and doubles the latency hiding
  static constexpr int kWarps = F8 ? 8 : (D == 256 ? 6 : kTcWarps);
  static constexpr int kWarpBudget = F8 ? 24 * 1024 : (D == 256 ? 32 * 1024 : 48 * 1024);  // a warp's stages
  static constexpr int kTileBytes = 16 * D * 2;         // 16-bit K (or V) bytes of one 16-token tile
  static constexpr int kTile8Bytes = 16 * D;            // fp8 K (or V) bytes of one tile
  static constexpr int kStageBytes = F8 ? 2 * kTile8Bytes : 2 * kTileBytes;  // K + V
  static constexpr int kScaleArea = F8 ? 1024 : 0;  // 8 stages x 128 bytes of scales
  static constexpr int kStages = kWarpBudget / kStageBytes < 8 ? kWarpBudget / kStageBytes : 8;
  static constexpr int kWarpBytes = kStages * kStageBytes + kScaleArea;
  static constexpr int kSmemBytes = kWarps * kWarpBytes + kWarps * kStages * 8 + 1024;
  static_assert(kStages >= 2, "need at least two stages");
  static_assert(kStageBytes % 1024 == 0 && kWarpBytes % 1024 == 0, "TMA tiles must stay 1024-byte aligned");
};

template <typename I>
__device__ __forceinline__ int64_t capped_len(const I* seq_lens, int b, int64_t cap) {
  const int64_t len = load_index(seq_lens, b);
  return len > cap ? cap : len;
}

// 16-token tiles of request b per KV head (0 for a request without tokens).
template <typename I>
__device__ __forceinline__ int request_tiles(const I* seq_lens, int b, int64_t cap) {
  const int64_t len = capped_len(seq_lens, b, cap);
  return len > 0 ? static_cast<int>((len + 15) >> 4) : 0;
}

// Warps that share the tile stream: every resident warp, or fewer when pages_per_split asks for
// about that many pages per warp, and never more than there are tiles.
__device__ __forceinline__ int64_t stream_warps(int64_t grid_warps, int64_t total, int32_t pages_per_split,
                                                int32_t block_size) {
  int64_t warps = grid_warps;
  if (pages_per_split > 0) {
    const int64_t per_warp = static_cast<int64_t>(pages_per_split) * (block_size >> 4);
    warps = min(warps, (total + per_warp - 1) / per_warp);
  }
  return min(warps, total);
}

// A (request, KV head) segment of the tile stream: its request, KV head, first tile, tile count.
struct Segment {
  int b, kvh, start, tiles;
};

// The segment after `c` in stream order: the next KV head of the same request, else KV head 0 of the
// next request with tokens (b == batch when the stream is exhausted).
template <typename I>
__device__ Segment next_segment(const Segment& c, const I* seq_lens, int batch, int num_kv_heads, int64_t cap) {
  Segment n = c;
  n.start = c.start + c.tiles;
  if (c.kvh + 1 < num_kv_heads) {
    n.kvh = c.kvh + 1;
    return n;
  }
  n.kvh = 0;
  for (int b = c.b + 1; b < batch; ++b) {
    const int t = request_tiles(seq_lens, b, cap);
    if (t > 0) {
      n.b = b;
      n.tiles = t;
      return n;
    }
  }
  n.b = batch;
  n.tiles = 0;
  return n;
}

// head_dim index of row r (0..15) of P.V m-tile k: natural for 16-bit pools; for fp8 pools the V^T
// fragments pair adjacent d-values (see the P.V loop): row r is d = 16k + 2(r & 7) + (r >> 3).
template <bool F8>
__device__ __forceinline__ int out_row_d(int k, int r) {
  if constexpr (F8) {
    return 16 * k + 2 * (r & 7) + (r >> 3);
  } else {
    return 16 * k + r;
  }
}

// Byte-permute selector for one ldmatrix.trans register of fp8 V: source bytes {t0 d0, t0 d1, t1 d0,
// t1 d1} (tokens t0, t1 of a lane; d-values d0, d1) become {t0 d0, t1 d0 | t0 d1, t1 d1}; selector
// nibble 4 takes a zero byte (the second operand) for a slot past the context.
__device__ __forceinline__ uint32_t fp8_token_pair_selector(bool v0, bool v1) {
  return (v0 ? 0x0u : 0x4u) | ((v1 ? 0x2u : 0x4u) << 4) | ((v0 ? 0x1u : 0x4u) << 8) | ((v1 ? 0x3u : 0x4u) << 12);
}

// Each warp owns a contiguous slice of the global tile stream and runs its own TMA pipeline over it:
// it issues the loads of tile i + NST after consuming tile i, crossing segment boundaries without
// draining. The slice and its first segment are derived in-kernel from seq_lens (no plan launch).
// At the end of every segment piece it writes the final output (piece == whole segment) or a
// partial that the segment's last finishing piece merges.
template <typename T, typename I, int D, bool F8 = false>
__global__ void __launch_bounds__(TcConfig<D, F8>::kWarps * 32, 1)
    decode_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                     const TcArgs<I> a) {
  // chained launches: resident before the previous kernel ends, and nothing is read before it completed --
  // except, with a.prefetch, the tables, lengths and pages (the caller guarantees that the previous kernel
  // does not write them), whose first loads then overlap that kernel's end
  if (!a.prefetch) pdl_wait();
  pdl_launch_dependents();
  using Cfg = TcConfig<D, F8>;
  // MMA operand type: the query/output type, or fp16 for fp8 pools (K/V widened exactly to f16)
  using TM = typename std::conditional<F8, __half, T>::type;
  constexpr int NST = Cfg::kStages;
  constexpr int NT = D / 16;  // m-tiles of the P.V product
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint8_t* wsm = smem + warp * Cfg::kWarpBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + Cfg::kWarps * Cfg::kWarpBytes) + warp * NST;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * Cfg::kWarps + warp;
  const int64_t grid_warps = static_cast<int64_t>(gridDim.x) * Cfg::kWarps;
  const int64_t cap = static_cast<int64_t>(a.max_blocks) * a.block_size;
  const int Hq = a.num_kv_heads * a.group;
  T* obase = static_cast<T*>(a.out);

  // ---- in-kernel plan: total tiles, this warp's slice, its first segment
  int64_t total = 0;
  for (int b = lane; b < a.batch; b += 32) {
    total += request_tiles(a.seq_lens, b, cap);
    if (gw == 0 && load_index(a.seq_lens, b) > cap) raise_device_error(a.error_flag, PKV_DEVERR_TABLE_TOO_SHORT);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) total += __shfl_xor_sync(0xffffffffu, total, off);
  total *= a.num_kv_heads;
  // requests without tokens produce zeros, spread over all warps of the grid (output: after the wait)
  auto zero_empty_requests = [&]() {
    for (int64_t b = gw; b < a.batch; b += grid_warps) {
      if (load_index(a.seq_lens, b) > 0) continue;
      for (int h = 0; h < Hq; ++h) {
        T* row = obase + b * a.o_sb + h * a.o_sh;
        for (int d = lane; d < D; d += 32) row[d] = Elem<T>::from_f(0.f);
      }
    }
  };
  if (!a.prefetch) zero_empty_requests();
  const int64_t warps = stream_warps(grid_warps, total, a.pages_per_split, a.block_size);
  if (gw >= warps) {
    if (a.prefetch) {
      pdl_wait();
      zero_empty_requests();
    }
    return;
  }
  const int64_t t0 = gw * total / warps;
  const int n = static_cast<int>((gw + 1) * total / warps - t0);

  Segment first{0, 0, 0, 0};
  {
    int64_t run = 0;
    for (int base = 0; base < a.batch; base += 32) {
      const int b = base + lane;
      const int tb = b < a.batch ? request_tiles(a.seq_lens, b, cap) : 0;
      const int64_t v = static_cast<int64_t>(tb) * a.num_kv_heads;
      int64_t incl = v;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const int64_t u = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += u;
      }
      const unsigned hit = __ballot_sync(0xffffffffu, run + incl > t0);
      if (hit != 0) {
        const int src = __ffs(hit) - 1;
        const int64_t excl = __shfl_sync(0xffffffffu, run + incl - v, src);
        const int tiles = __shfl_sync(0xffffffffu, tb, src);
        const int kvh = static_cast<int>((t0 - excl) / tiles);
        first = Segment{base + src, kvh, static_cast<int>(excl + static_cast<int64_t>(kvh) * tiles), tiles};
        break;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
    }
  }

  if (lane == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
#pragma unroll
    for (int s = 0; s < NST; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  const uint64_t policy = policy_evict_first();
  const int g = lane >> 2, t = lane & 3;
  const int tiles_per_page = a.block_size >> 4;
  const int v_tok = (lane & 7) + ((lane >> 4) << 3);
  const int v_half = (lane >> 3) & 1;
  const T* qbase = static_cast<const T*>(a.q);

  // ---- producer cursor
  Segment pseg = first;
  int pj = static_cast<int>(t0 - pseg.start);
  const I* ptab = a.tables + static_cast<int64_t>(pseg.b) * a.table_stride;
  int64_t ppages = (capped_len(a.seq_lens, pseg.b, cap) + a.block_size - 1) / a.block_size;
  int tbl_base = ((pj / tiles_per_page) >> 5) << 5;
  int64_t tbl = (tbl_base + lane < ppages) ? load_index(ptab, tbl_base + lane) : -1;
  uint32_t bad_bits = 0, pending_bits = 0, phase_bits = 0;

  auto issue = [&](int i) {
    const int page_local = pj / tiles_per_page;
    const int sub = pj - page_local * tiles_per_page;
    if (page_local - tbl_base >= 32) {
      tbl_base = (page_local >> 5) << 5;
      tbl = (tbl_base + lane < ppages) ? load_index(ptab, tbl_base + lane) : -1;
    }
    const int64_t page = __shfl_sync(0xffffffffu, tbl, page_local - tbl_base);
    const int s = i % NST;
    const bool ok = page >= 0 && page < a.num_pages;
    if (ok) bad_bits &= ~(1u << s); else bad_bits |= (1u << s);
    pending_bits |= (1u << s);
    if (lane == 0) {
      if (ok) {
        uint8_t* kst = wsm + s * Cfg::kStageBytes;
        mbar_arrive_expect_tx(&bars[s], Cfg::kStageBytes + (F8 ? 128 : 0));
        const int row = static_cast<int>(page) * a.rows_per_page + pseg.kvh * a.rows_per_head + sub * 16;
        if constexpr (F8) {
          tma_load_3d(kst, &kmap, &bars[s], 0, row, 0, policy);
          tma_load_3d(kst + Cfg::kTile8Bytes, &vmap, &bars[s], 0, row, 0, policy);
          const int64_t sofs = page * a.scale_sp + static_cast<int64_t>(pseg.kvh) * a.scale_sh + sub * 16;
          uint8_t* scl = wsm + NST * Cfg::kStageBytes + s * 128;
          bulk_load(scl, a.k_scales + sofs, 64, &bars[s]);
          bulk_load(scl + 64, a.v_scales + sofs, 64, &bars[s]);
        } else {
          tma_load_3d(kst, &kmap, &bars[s], 0, row, 0, policy);
          tma_load_3d(kst + Cfg::kTileBytes, &vmap, &bars[s], 0, row, 0, policy);
        }
      } else {
        mbar_arrive(&bars[s]);
      }
    }
    if (++pj == pseg.tiles) {  // next segment of the stream
      const int prev_b = pseg.b;
      pseg = next_segment(pseg, a.seq_lens, a.batch, a.num_kv_heads, cap);
      pj = 0;
      if (pseg.b < a.batch) {
        if (pseg.b != prev_b) {
          ptab = a.tables + static_cast<int64_t>(pseg.b) * a.table_stride;
          ppages = (capped_len(a.seq_lens, pseg.b, cap) + a.block_size - 1) / a.block_size;
        }
        tbl_base = 0;
        tbl = lane < ppages ? load_index(ptab, lane) : -1;
      }
    }
  };

  const int npro = n < NST ? n : NST;
  for (int i = 0; i < npro; ++i) issue(i);
  if (a.prefetch) {  // the query, the outputs and the workspace only after the previous kernel completed
    pdl_wait();
    zero_empty_requests();
  }

  // ---- consumer cursor
  Segment cseg = first;
  int cj = static_cast<int>(t0 - cseg.start);
  int64_t clen = 0;
  bool piece_bad = false, piece_first = true;
  uint32_t qf[D / 64][2][4];
  float m0 = kNegInf, m1 = kNegInf, l0 = 0.f, l1 = 0.f;
  float acc[NT][4];

  for (int i = 0; i < n; ++i) {
    if (i == 0 || cj == 0) {  // a piece starts: this segment's query heads, fresh softmax state
      piece_first = i == 0;
      clen = capped_len(a.seq_lens, cseg.b, cap);
      const bool hv = g < a.group;
      const T* qp = qbase + static_cast<int64_t>(cseg.b) * a.q_sb + (cseg.kvh * a.group + (hv ? g : 0)) * a.q_sh;
#pragma unroll
      for (int bx = 0; bx < D / 64; ++bx) {
#pragma unroll
        for (int uu = 0; uu < 2; ++uu) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (hv) v = *reinterpret_cast<const uint4*>(qp + bx * 64 + 8 * (2 * t + uu));
          if constexpr (F8 && !std::is_same<T, __half>::value) {  // the MMA runs in fp16
            const float2 f0 = unpack2<T>(v.x), f1 = unpack2<T>(v.y), f2 = unpack2<T>(v.z), f3 = unpack2<T>(v.w);
            v = make_uint4(pack2<__half>(f0.x, f0.y), pack2<__half>(f1.x, f1.y), pack2<__half>(f2.x, f2.y),
                           pack2<__half>(f3.x, f3.y));
          }
          qf[bx][uu][0] = v.x; qf[bx][uu][1] = v.y; qf[bx][uu][2] = v.z; qf[bx][uu][3] = v.w;
        }
      }
      m0 = kNegInf; m1 = kNegInf; l0 = 0.f; l1 = 0.f;
#pragma unroll
      for (int k = 0; k < NT; ++k) acc[k][0] = acc[k][1] = acc[k][2] = acc[k][3] = 0.f;
      piece_bad = false;
    }
    const int s = i % NST;
    const bool landed = mbar_wait_bounded(&bars[s], (phase_bits >> s) & 1u, kWaitTimeoutNs);
    if (!__all_sync(0xffffffffu, landed)) {
      // A load never completed: report, give in-flight copies a bounded chance to land, stop.
      if (lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
      for (int r = 0; r < NST; ++r) {
        if (r != s && (pending_bits & (1u << r))) mbar_wait_bounded(&bars[r], (phase_bits >> r) & 1u, kWaitTimeoutNs);
      }
      return;
    }
    phase_bits ^= (1u << s);
    pending_bits &= ~(1u << s);
    if (bad_bits & (1u << s)) {
      piece_bad = true;
    } else {
      const int64_t rem = clen - static_cast<int64_t>(cj) * 16;
      const int nv = rem < 16 ? static_cast<int>(rem) : 16;
      const uint32_t kb = smem_u32(wsm + s * Cfg::kStageBytes);
      const uint32_t vb = kb + (F8 ? Cfg::kTile8Bytes : Cfg::kTileBytes);
      // ---- S^T = K . Q^T
      float c[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      const uint32_t sw = static_cast<uint32_t>(g & 7);
      if constexpr (F8) {
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx) {
          // elements 64 bx + 16 t .. + 15 of rows g, g + 8: one 16-byte unit of the fp8 tile's 128-element
          // boxes, widened exactly to f16; uu selects its half
          const uint32_t off = (bx >> 1) * 2048 + ((((bx & 1) * 4 + t) ^ sw) << 4);
          const uint4 rg = lds128(kb + off + g * 128), rh = lds128(kb + off + (g + 8) * 128);
#pragma unroll
          for (int uu = 0; uu < 2; ++uu) {
            uint4 ka, kc;
            e4m3x4_to_f16x2(uu ? rg.z : rg.x, ka.x, ka.y);
            e4m3x4_to_f16x2(uu ? rg.w : rg.y, ka.z, ka.w);
            e4m3x4_to_f16x2(uu ? rh.z : rh.x, kc.x, kc.y);
            e4m3x4_to_f16x2(uu ? rh.w : rh.y, kc.z, kc.w);
            mma_16816<TM>(c[uu], ka.x, kc.x, ka.y, kc.y, qf[bx][uu][0], qf[bx][uu][1]);
            mma_16816<TM>(c[uu], ka.z, kc.z, ka.w, kc.w, qf[bx][uu][2], qf[bx][uu][3]);
          }
        }
      } else {
#pragma unroll
        for (int bx = 0; bx < D / 64; ++bx) {
#pragma unroll
          for (int uu = 0; uu < 2; ++uu) {
            const uint32_t chunk = ((2 * t + uu) ^ sw) << 4;
            const uint4 ka = lds128(kb + bx * 2048 + g * 128 + chunk);
            const uint4 kc = lds128(kb + bx * 2048 + (g + 8) * 128 + chunk);
            mma_16816<TM>(c[uu], ka.x, kc.x, ka.y, kc.y, qf[bx][uu][0], qf[bx][uu][1]);
            mma_16816<TM>(c[uu], ka.z, kc.z, ka.w, kc.w, qf[bx][uu][2], qf[bx][uu][3]);
          }
        }
      }
      float sc0 = a.scale_log2, sc1 = a.scale_log2;  // score scale of tokens g, g + 8
      float vs0 = 1.f, vs1 = 1.f;                    // P scale of tokens g, g + 8
      if constexpr (F8) {  // dequantisation: per-token scales
        const float* scl = reinterpret_cast<const float*>(wsm + NST * Cfg::kStageBytes + s * 128);
        sc0 *= scl[g];
        sc1 *= scl[g + 8];
        vs0 = scl[16 + g];
        vs1 = scl[16 + g + 8];
      }
      float s0 = (c[0][0] + c[1][0]) * sc0;  // token g,   head 2t
      float s1 = (c[0][1] + c[1][1]) * sc0;  // token g,   head 2t+1
      float s2 = (c[0][2] + c[1][2]) * sc1;  // token g+8, head 2t
      float s3 = (c[0][3] + c[1][3]) * sc1;  // token g+8, head 2t+1
      if (nv < 16) {  // a partial tile (warp-uniform): slots past the context take no part, and their P
                      // scale is 0 so that a never-written scale cannot reach O
        if (g >= nv) { s0 = kNegInf; s1 = kNegInf; vs0 = 0.f; }
        if (g + 8 >= nv) { s2 = kNegInf; s3 = kNegInf; vs1 = 0.f; }
      }
      // ---- online softmax over the tile's tokens
      float mx0 = fmaxf(s0, s2), mx1 = fmaxf(s1, s3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
      const float base0 = mn0 == kNegInf ? 0.f : mn0;
      const float base1 = mn1 == kNegInf ? 0.f : mn1;
      const float alpha0 = fast_exp2(m0 - base0), alpha1 = fast_exp2(m1 - base1);
      const float p0 = fast_exp2(s0 - base0), p1 = fast_exp2(s1 - base1);
      const float p2 = fast_exp2(s2 - base0), p3 = fast_exp2(s3 - base1);
      l0 = l0 * alpha0 + p0 + p2;
      l1 = l1 * alpha1 + p1 + p3;
      m0 = mn0;
      m1 = mn1;
      if (__any_sync(0xffffffffu, alpha0 != 1.f || alpha1 != 1.f)) {
#pragma unroll
        for (int k = 0; k < NT; ++k) {
          acc[k][0] *= alpha0; acc[k][1] *= alpha1; acc[k][2] *= alpha0; acc[k][3] *= alpha1;
        }
      }
      // ---- P^T as the B fragment (head g, tokens 2t.. / 2t+8..). bf16 keeps only 8 mantissa bits,
      // so P is carried as hi + lo bf16 parts (two P.V products) and stays fp32-accurate.
      const float q0 = p0 * vs0, q1 = p1 * vs0, q2 = p2 * vs1, q3 = p3 * vs1;  // V dequantisation (fp8)
      const uint32_t ph0 = pack2<TM>(q0, q1), ph1 = pack2<TM>(q2, q3);
      const uint32_t pb0 = movmatrix_trans(ph0);
      const uint32_t pb1 = movmatrix_trans(ph1);
      uint32_t pl0 = 0, pl1 = 0;
      if constexpr (kSplitP<TM>) {
        const float2 h01 = unpack2<TM>(ph0), h23 = unpack2<TM>(ph1);
        pl0 = movmatrix_trans(pack2<TM>(q0 - h01.x, q1 - h01.y));
        pl1 = movmatrix_trans(pack2<TM>(q2 - h23.x, q3 - h23.y));
      }
      // ---- O^T += V^T . P^T (V of empty slots zeroed so that 0 * garbage cannot produce NaN)
      if constexpr (F8) {
        // V^T fragments straight from the fp8 tile. ldmatrix.trans over b16 pairs of fp8 bytes gives lane
        // (g, t) the bytes {token 2t, 2t + 1} x {d 16u + 2g, 16u + 2g + 1} of a 16-byte unit u; one byte
        // permute regroups them by d (and zeroes the bytes of slots past the context), and the widening
        // gives exact f16 pairs. Row r of m-tile u is d = 16u + 2(r & 7) + (r >> 3).
        const uint32_t sel_a = fp8_token_pair_selector(2 * t < nv, 2 * t + 1 < nv);
        const uint32_t sel_b = fp8_token_pair_selector(2 * t + 8 < nv, 2 * t + 9 < nv);
        const int ltok = (lane & 7) + (lane & 8);  // row addressed by this lane: tokens 0-7, 8-15, 0-7, 8-15
        const int lunit = lane >> 4;               // ... of unit 2j (lanes 0-15) or 2j + 1 (lanes 16-31)
#pragma unroll
        for (int j = 0; j < D / 32; ++j) {
          const uint32_t addr = vb + (j >> 2) * 2048 + ltok * 128 + ((((2 * j + lunit) & 7) ^ (ltok & 7)) << 4);
          uint32_t r0, r1, r2, r3;
          ldsm_x4_trans(addr, r0, r1, r2, r3);
          uint32_t a0, a1, a2, a3;
          e4m3x4_to_f16x2(__byte_perm(r0, 0u, sel_a), a0, a1);
          e4m3x4_to_f16x2(__byte_perm(r1, 0u, sel_b), a2, a3);
          mma_16816<TM>(acc[2 * j], a0, a1, a2, a3, pb0, pb1);
          e4m3x4_to_f16x2(__byte_perm(r2, 0u, sel_a), a0, a1);
          e4m3x4_to_f16x2(__byte_perm(r3, 0u, sel_b), a2, a3);
          mma_16816<TM>(acc[2 * j + 1], a0, a1, a2, a3, pb0, pb1);
        }
      } else {
        const uint32_t mlo = (2 * t < nv ? 0x0000ffffu : 0u) | (2 * t + 1 < nv ? 0xffff0000u : 0u);
        const uint32_t mhi = (2 * t + 8 < nv ? 0x0000ffffu : 0u) | (2 * t + 9 < nv ? 0xffff0000u : 0u);
#pragma unroll
        for (int k = 0; k < NT; ++k) {
          const int chunk = 2 * k + v_half;
          const uint32_t addr = vb + (chunk >> 3) * 2048 + v_tok * 128 + (((chunk & 7) ^ (v_tok & 7)) << 4);
          uint32_t a0, a1, a2, a3;
          ldsm_x4_trans(addr, a0, a1, a2, a3);
          if (nv < 16) { a0 &= mlo; a1 &= mlo; a2 &= mhi; a3 &= mhi; }
          mma_16816<TM>(acc[k], a0, a1, a2, a3, pb0, pb1);
          if constexpr (kSplitP<TM>) mma_16816<TM>(acc[k], a0, a1, a2, a3, pl0, pl1);
        }
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (i + NST < n) issue(i + NST);
    ++cj;

    if (cj < cseg.tiles && i + 1 < n) continue;
    // ---- the piece ends: final output, or a partial merged by the segment's last piece
    if (piece_bad && lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_PAGE_OUT_OF_RANGE);
    float lt0 = l0, lt1 = l1;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      lt0 += __shfl_xor_sync(0xffffffffu, lt0, off);
      lt1 += __shfl_xor_sync(0xffffffffu, lt1, off);
    }
    const int h0 = 2 * t, h1 = 2 * t + 1;
    const int G = a.group;
    const int b = cseg.b;
    const int qh0 = cseg.kvh * G;
    const int64_t wa = warp_of_tile(cseg.start, total, warps);
    const int pieces = static_cast<int>(warp_of_tile(cseg.start + cseg.tiles - 1, total, warps) - wa + 1);
    if (pieces <= 1) {
      const float inv0 = lt0 > 0.f ? 1.f / lt0 : 0.f;
      const float inv1 = lt1 > 0.f ? 1.f / lt1 : 0.f;
      T* o0 = obase + b * a.o_sb + (qh0 + h0) * a.o_sh;
      T* o1 = obase + b * a.o_sb + (qh0 + h1) * a.o_sh;
#pragma unroll
      for (int k = 0; k < NT; ++k) {
        const int d0 = out_row_d<F8>(k, g), d1 = out_row_d<F8>(k, g + 8);
        if (h0 < G) {
          o0[d0] = Elem<T>::from_f(acc[k][0] * inv0);
          o0[d1] = Elem<T>::from_f(acc[k][2] * inv0);
        }
        if (h1 < G) {
          o1[d0] = Elem<T>::from_f(acc[k][1] * inv1);
          o1[d1] = Elem<T>::from_f(acc[k][3] * inv1);
        }
      }
    } else {
      const int slot = static_cast<int>(2 * gw) + (piece_first ? 0 : 1);
      if (g == 0) {
        if (h0 < G) a.ws.part_ml[slot * G + h0] = make_float2(m0, lt0);
        if (h1 < G) a.ws.part_ml[slot * G + h1] = make_float2(m1, lt1);
      }
      float* pa0 = a.ws.part_acc + (static_cast<int64_t>(slot) * G + h0) * D;
      float* pa1 = a.ws.part_acc + (static_cast<int64_t>(slot) * G + h1) * D;
#pragma unroll
      for (int k = 0; k < NT; ++k) {
        const int d0 = out_row_d<F8>(k, g), d1 = out_row_d<F8>(k, g + 8);
        if (h0 < G) { pa0[d0] = acc[k][0]; pa0[d1] = acc[k][2]; }
        if (h1 < G) { pa1[d0] = acc[k][1]; pa1[d1] = acc[k][3]; }
      }
    }
    if (cj == cseg.tiles && i + 1 < n) {  // the stream continues in the next segment
      cseg = next_segment(cseg, a.seq_lens, a.batch, a.num_kv_heads, cap);
      cj = 0;
    }
  }
}


// Merges the partials of every segment the tensor-core kernel split over several warps. Block
// (segment, column chunk): warp h merges query head h of the segment over 128 columns of head_dim
// (one float4 per lane), reading the pieces eight at a time. It repeats the stream arithmetic of the
// attention kernel (same tile counts, same warp count) to find which warps wrote the pieces: piece j
// came from warp wa + j, slot 2 * (wa + j), except that the first piece is in slot 2 * wa + 1 when
// the segment was not the first one of warp wa's slice.
template <typename T, typename I, int D>
__global__ void __launch_bounds__(256) decode_tc_merge_kernel(const TcArgs<I> a, int64_t grid_warps) {
  __shared__ int64_t s_red[2][8];
  // the next kernel may become resident now (it waits for this one before reading what this writes)
  pdl_launch_dependents();
  pdl_wait();  // the partials come from decode_tc_kernel
  const int seg = blockIdx.x;
  const int b = seg / a.num_kv_heads, kvh = seg - b * a.num_kv_heads;
  const int64_t cap = static_cast<int64_t>(a.max_blocks) * a.block_size;
  const int tiles = request_tiles(a.seq_lens, b, cap);
  if (tiles == 0) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int64_t total = 0, before = 0;
  for (int r = threadIdx.x; r < a.batch; r += blockDim.x) {
    const int64_t tr = request_tiles(a.seq_lens, r, cap);
    total += tr;
    if (r < b) before += tr;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    total += __shfl_xor_sync(0xffffffffu, total, off);
    before += __shfl_xor_sync(0xffffffffu, before, off);
  }
  if (lane == 0) { s_red[0][warp] = total; s_red[1][warp] = before; }
  __syncthreads();
  total = 0;
  before = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) { total += s_red[0][w]; before += s_red[1][w]; }
  total *= a.num_kv_heads;
  const int64_t warps = stream_warps(grid_warps, total, a.pages_per_split, a.block_size);
  const int64_t start = before * a.num_kv_heads + static_cast<int64_t>(kvh) * tiles;
  const int64_t wa = warp_of_tile(start, total, warps);
  const int pieces = static_cast<int>(warp_of_tile(start + tiles - 1, total, warps) - wa + 1);
  if (pieces <= 1) return;
  const bool first_is_second = wa * total / warps < start;
  const int G = a.group;
  const int h = warp;
  const int col = blockIdx.y * 128 + lane * 4;
  if (h >= G) return;  // warp-uniform; lanes past head_dim stay for the shuffles below
  auto slot_of = [&](int j) { return static_cast<int>(2 * (wa + j)) + ((j == 0 && first_is_second) ? 1 : 0); };
  float mx = kNegInf, lsum = 0.f;
  for (int j = lane; j < pieces; j += 32) {
    const float2 ml = a.ws.part_ml[slot_of(j) * G + h];
    const float mn = fmaxf(mx, ml.x);
    const float base = mn == kNegInf ? 0.f : mn;
    lsum = lsum * fast_exp2(mx - base) + ml.y * fast_exp2(ml.x - base);
    mx = mn;
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float om = __shfl_xor_sync(0xffffffffu, mx, off);
    const float ol = __shfl_xor_sync(0xffffffffu, lsum, off);
    const float mn = fmaxf(mx, om);
    const float base = mn == kNegInf ? 0.f : mn;
    lsum = lsum * fast_exp2(mx - base) + ol * fast_exp2(om - base);
    mx = mn;
  }
  const float base = mx == kNegInf ? 0.f : mx;
  const float inv = lsum > 0.f ? 1.f / lsum : 0.f;
  if (col >= D) return;
  float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int j0 = 0; j0 < pieces; j0 += 8) {
    float4 x[8];
    float w[8];
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      const int j = j0 + u;
      if (j < pieces) {
        const int slot = slot_of(j);
        w[u] = fast_exp2(a.ws.part_ml[slot * G + h].x - base) * inv;
        x[u] = *reinterpret_cast<const float4*>(a.ws.part_acc + (static_cast<int64_t>(slot) * G + h) * D + col);
      } else {
        w[u] = 0.f;
        x[u] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
    }
#pragma unroll
    for (int u = 0; u < 8; ++u) {
      o.x = fmaf(w[u], x[u].x, o.x); o.y = fmaf(w[u], x[u].y, o.y);
      o.z = fmaf(w[u], x[u].z, o.z); o.w = fmaf(w[u], x[u].w, o.w);
    }
  }
  T* orow = static_cast<T*>(a.out) + b * a.o_sb + (kvh * G + h) * a.o_sh + col;
  uint2 packed;
  packed.x = pack2<T>(o.x, o.y);
  packed.y = pack2<T>(o.z, o.w);
  *reinterpret_cast<uint2*>(orow) = packed;
}

// ---- generic CUDA-core kernel ------------------------------------------------------------------------------
template <typename I>
struct GenArgs {
  const void* q;
  int64_t q_sb, q_sh;
  const void* kpool;
  const void* vpool;
  const void* const* kptrs;  // per-request pools (reference batched layout) when non-null
  const void* const* vptrs;
  const int64_t* row_pages;  // per-request physical page counts in that mode
  int64_t pool_sb;           // batch stride of a pool with a batch dimension (elements)
  int64_t num_pages, block_size, head_dim;
  int64_t sp, sh, ss;  // pool strides (elements)
  const I* tables;
  int64_t table_stride, max_blocks;
  const I* seq_lens;
  int64_t uniform_len;
  int32_t batch, num_kv_heads, group;
  float scale_log2;
  Workspace ws;  // ws.units == nullptr: one CTA per (request, KV head), no split
  void* out;
  int64_t o_sb, o_sh;
  int32_t* error_flag;
};

template <typename T, typename I, int MAXK>
__global__ void __launch_bounds__(kGenThreads) decode_generic_kernel(const GenArgs<I> a) {
  constexpr int kWarps = kGenThreads / 32;
  __shared__ float s_m[kWarps], s_l[kWarps];
  __shared__ int s_unit;
  __shared__ int s_last;
  extern __shared__ float s_acc[];  // [kWarps][head_dim]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = static_cast<int>(a.head_dim);
  const T* qbase = static_cast<const T*>(a.q);
  T* obase = static_cast<T*>(a.out);
  const bool planned = a.ws.units != nullptr;
  const int num_units = planned ? a.ws.hdr->num_units : a.batch * a.num_kv_heads;
  const int pps = planned ? a.ws.hdr->pages_per_split : 0;
  int iter = 0;
  while (true) {
    int u;
    if (planned) {
      if (threadIdx.x == 0) s_unit = atomicAdd(&a.ws.hdr->unit_counter, 1);
      __syncthreads();
      u = s_unit;
      __syncthreads();
    } else {
      u = blockIdx.x + iter * gridDim.x;
      ++iter;
    }
    if (u >= num_units) break;
    int b, kvh, split, page_begin, page_end;
    int64_t len = request_len(a.seq_lens, a.uniform_len, u / a.num_kv_heads);
    if (planned) {
      const int4 unit = a.ws.units[u];
      b = unit.x; kvh = unit.y & 255; split = unit.y >> 8; page_begin = unit.z; page_end = unit.w;
      len = request_len(a.seq_lens, a.uniform_len, b);
    } else {
      b = u / a.num_kv_heads; kvh = u - b * a.num_kv_heads; split = 0; page_begin = 0;
      page_end = static_cast<int>(a.max_blocks);
    }
    const int64_t cap = a.max_blocks * a.block_size;
    if (len > cap) {
      if (threadIdx.x == 0 && !planned) raise_device_error(a.error_flag, PKV_DEVERR_TABLE_TOO_SHORT);
      len = cap;
    }
    const int64_t tok_begin = static_cast<int64_t>(page_begin) * a.block_size;
    const int64_t tok_end = min(static_cast<int64_t>(page_end) * a.block_size, len);
    const int ns = planned ? static_cast<int>(((len + a.block_size - 1) / a.block_size + pps - 1) / pps) : 1;
    const char* kp;
    const char* vp;
    int64_t num_pages = a.num_pages, sh = a.sh;
    const int es = sizeof(T);
    if (a.kptrs != nullptr) {
      kp = static_cast<const char*>(a.kptrs[b]);
      vp = static_cast<const char*>(a.vptrs[b]);
      num_pages = a.row_pages[b];
      // the reference's (1, heads, pages, block_size, D) pools: the head stride follows the page count;
      // native (pages, kv heads, block_size, D) pools pass their head stride
      if (sh == 0) sh = num_pages * a.block_size * a.head_dim;
    } else {
      kp = static_cast<const char*>(a.kpool) + b * a.pool_sb * es;
      vp = static_cast<const char*>(a.vpool) + b * a.pool_sb * es;
    }
    const I* trow = a.tables + b * a.table_stride;
    const int qh0 = kvh * a.group;
    bool bad = false;

    if (len <= 0) {
      // only reachable without a plan (the plan zeroes empty rows itself)
      for (int i = threadIdx.x; i < a.group * D; i += blockDim.x) {
        const int h = i / D, d = i - h * D;
        obase[b * a.o_sb + (qh0 + h) * a.o_sh + d] = Elem<T>::from_f(0.f);
      }
      continue;
    }

    for (int h = 0; h < a.group; ++h) {
      float q[MAXK], acc[MAXK];
      const T* qrow = qbase + b * a.q_sb + (qh0 + h) * a.q_sh;
#pragma unroll
      for (int k = 0; k < MAXK; ++k) {
        const int d = k * 32 + lane;
        q[k] = d < D ? Elem<T>::to_f(qrow[d]) : 0.f;
        acc[k] = 0.f;
      }
      float m = kNegInf, l = 0.f;
      for (int64_t tok = tok_begin + warp; tok < tok_end; tok += kWarps) {
        const int64_t logical = tok / a.block_size;
        const int64_t page = load_index(trow, logical);
        if (page < 0 || page >= num_pages) {
          bad = true;
          continue;
        }
        const int64_t off = (page * a.sp + kvh * sh + (tok - logical * a.block_size) * a.ss) * es;
        const T* krow = reinterpret_cast<const T*>(kp + off);
        const T* vrow = reinterpret_cast<const T*>(vp + off);
        float part = 0.f;
#pragma unroll
        for (int k = 0; k < MAXK; ++k) {
          const int d = k * 32 + lane;
          if (d < D) part = fmaf(q[k], Elem<T>::to_f(krow[d]), part);
        }
#pragma unroll
        for (int off2 = 16; off2 > 0; off2 >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off2);
        const float sc = part * a.scale_log2;
        const float mn = fmaxf(m, sc);
        const float base = mn == kNegInf ? 0.f : mn;
        const float alpha = fast_exp2(m - base);
        const float p = fast_exp2(sc - base);
        l = l * alpha + p;
        m = mn;
#pragma unroll
        for (int k = 0; k < MAXK; ++k) {
          const int d = k * 32 + lane;
          const float v = d < D ? Elem<T>::to_f(vrow[d]) : 0.f;
          acc[k] = fmaf(p, v, acc[k] * alpha);
        }
      }
      // merge the warps' partial states
      if (lane == 0) { s_m[warp] = m; s_l[warp] = l; }
#pragma unroll
      for (int k = 0; k < MAXK; ++k) {
        const int d = k * 32 + lane;
        if (d < D) s_acc[warp * D + d] = acc[k];
      }
      __syncthreads();
      float mt = kNegInf;
#pragma unroll
      for (int w = 0; w < kWarps; ++w) mt = fmaxf(mt, s_m[w]);
      const float base = mt == kNegInf ? 0.f : mt;
      float lt = 0.f, wts[kWarps];
#pragma unroll
      for (int w = 0; w < kWarps; ++w) {
        wts[w] = fast_exp2(s_m[w] - base);
        lt += s_l[w] * wts[w];
      }
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      for (int d = threadIdx.x; d < D; d += blockDim.x) {
        float o = 0.f;
#pragma unroll
        for (int w = 0; w < kWarps; ++w) o += wts[w] * s_acc[w * D + d];
        if (ns <= 1) {
          obase[b * a.o_sb + (qh0 + h) * a.o_sh + d] = Elem<T>::from_f(o * inv);
        } else {
          a.ws.part_acc[(static_cast<int64_t>(u) * a.group + h) * D + d] = o;
        }
      }
      if (ns > 1 && threadIdx.x == 0) a.ws.part_ml[u * a.group + h] = make_float2(mt, lt);
      __syncthreads();
    }
    if (__syncthreads_or(bad) && threadIdx.x == 0) raise_device_error(a.error_flag, PKV_DEVERR_PAGE_OUT_OF_RANGE);
    if (ns > 1) {
      __threadfence();
      __syncthreads();
      if (threadIdx.x == 0) s_last = atomicAdd(&a.ws.counters[b * a.num_kv_heads + kvh], 1) == ns - 1;
      __syncthreads();
      if (s_last) {
        __threadfence();
        if (warp == 0) merge_splits_warp<T>(a.ws, u - split, ns, a.group, D, obase, a.o_sb, a.o_sh, b, qh0, lane);
        if (threadIdx.x == 0) a.ws.counters[b * a.num_kv_heads + kvh] = 0;
      }
      __syncthreads();
    }
  }
}

// ---- standalone LSE merge ------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256) lse_merge_kernel(const float* part_out, const float* part_lse, int64_t parts,
                                                        int64_t rows, int64_t D, T* out, int64_t o_sr,
                                                        float* out_lse) {
  const int64_t row = blockIdx.x;
  if (row >= rows) return;
  float mx = kNegInf;
  for (int64_t s = 0; s < parts; ++s) mx = fmaxf(mx, part_lse[s * rows + row]);
  const float base = mx == kNegInf ? 0.f : mx;
  float tot = 0.f;
  for (int64_t s = 0; s < parts; ++s) tot += expf(part_lse[s * rows + row] - base);
  const float inv = tot > 0.f ? 1.f / tot : 0.f;
  for (int64_t d = threadIdx.x; d < D; d += blockDim.x) {
    float o = 0.f;
    for (int64_t s = 0; s < parts; ++s) {
      const float w = expf(part_lse[s * rows + row] - base);
      if (w > 0.f) o += w * part_out[(s * rows + row) * D + d];
    }
    out[row * o_sr + d] = Elem<T>::from_f(o * inv);
  }
  if (out_lse != nullptr && threadIdx.x == 0) out_lse[row] = tot > 0.f ? base + logf(tot) : kNegInf;
}

// ---- host helpers --------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }
  });
  return fn;
}

// The pool seen as a 3-D tensor {64 elements, rows, head_dim / 64 chunks} with the chunk dimension
// outermost (stride 128 bytes) and rows in the middle (stride head_dim * 2 bytes): one box
// {64, 16, head_dim / 64} is a whole 16-token tile of one KV head, landing in shared memory as
// head_dim/64 consecutive 16-row x 128-byte blocks with the 128-byte swizzle.
int encode_pool_map(CUtensorMap* map, const void* pool, int dtype, int64_t head_dim, int64_t rows) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return PKV_ERR_CUDA;
  }
  cuuint64_t dims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(head_dim / 64)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim * 2), 128};
  cuuint32_t box[3] = {64, 16, static_cast<cuuint32_t>(head_dim / 64)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, dtype == PKV_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                  const_cast<void*>(pool), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

// FP8 pool viewed as (128 bytes, rows, head_dim / 128): one box = a whole 16-token tile of 128-byte
// swizzled boxes.
int encode_pool_map_fp8(CUtensorMap* map, const void* pool, int64_t head_dim, int64_t rows) {
  auto fn = tensor_map_encoder();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return PKV_ERR_CUDA;
  }
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(head_dim / 128)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim), 128};
  cuuint32_t box[3] = {128, 16, static_cast<cuuint32_t>(head_dim / 128)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(pool), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

int device_sms() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

Workspace carve(void* base, const WsLayout& w) {
  char* p = static_cast<char*>(base);
  return Workspace{reinterpret_cast<WsHeader*>(p), reinterpret_cast<int32_t*>(p + w.counters_off),
                   reinterpret_cast<int4*>(p + w.units_off), reinterpret_cast<float2*>(p + w.ml_off),
                   reinterpret_cast<float*>(p + w.acc_off), static_cast<int32_t>(w.max_units)};
}

// Launches the tensor-core kernel on as many CTAs as stay resident (capped by kMaxStreamWarps).
template <typename T, typename I, int D, bool F8 = false>
int launch_tc(const TcArgs<I>& a, const CUtensorMap& km, const CUtensorMap& vm, cudaStream_t s) {
  using Cfg = TcConfig<D, F8>;
  auto kern = decode_tc_kernel<T, I, D, F8>;
  int per_sm = 1;
  const cudaError_t e0 =
      prepare_kernel(reinterpret_cast<const void*>(kern), Cfg::kSmemBytes, Cfg::kWarps * 32, &per_sm);
  if (e0 != cudaSuccess) return cuda_status(e0, "decode_tc_kernel smem attribute / occupancy");
  const int grid = std::min(device_sms() * per_sm, kMaxStreamWarps / Cfg::kWarps);
  const dim3 merge_grid(static_cast<unsigned>(a.batch) * a.num_kv_heads, (D + 127) / 128);
  const int64_t grid_warps = static_cast<int64_t>(grid) * Cfg::kWarps;
  if (!a.chained) {
    kern<<<grid, Cfg::kWarps * 32, Cfg::kSmemBytes, s>>>(km, vm, a);
    int st = cuda_status(cudaGetLastError(), "decode_tc_kernel launch");
    if (st != PKV_OK) return st;
    decode_tc_merge_kernel<T, I, D><<<merge_grid, 256, 0, s>>>(a, grid_warps);
    return cuda_status(cudaGetLastError(), "decode_tc_merge_kernel launch");
  }
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(Cfg::kWarps * 32);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = s;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, km, vm, a);
  if (e != cudaSuccess) return cuda_status(e, "decode_tc_kernel launch");
  cfg.gridDim = merge_grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  e = cudaLaunchKernelEx(&cfg, decode_tc_merge_kernel<T, I, D>, a, grid_warps);
  return cuda_status(e, "decode_tc_merge_kernel launch");
}

template <typename T, typename I>
int launch_generic(const GenArgs<I>& a, int64_t grid, cudaStream_t s) {
  const size_t smem = static_cast<size_t>(kGenThreads / 32) * a.head_dim * sizeof(float);
  if (a.head_dim <= 256) {
    decode_generic_kernel<T, I, 8><<<grid, kGenThreads, smem, s>>>(a);
  } else {
    decode_generic_kernel<T, I, 32><<<grid, kGenThreads, smem, s>>>(a);
  }
  return cuda_status(cudaGetLastError(), "decode_generic_kernel launch");
}

template <typename I>
int run_decode(const void* query, int64_t q_sb, int64_t q_sh, const void* key_pool, const void* value_pool,
               int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim, int64_t sp, int64_t sh,
               int64_t ss, const void* tables, int64_t table_stride, int64_t max_blocks, const void* seq_lens,
               int64_t batch, int64_t num_q_heads, float scale, int64_t pages_per_split, void* workspace,
               int64_t workspace_bytes, void* output, int64_t o_sb, int64_t o_sh, int dtype, int flags,
               int32_t* error_flag, cudaStream_t stream) {
  const int es = dtype_size(dtype);
  const int64_t group = num_q_heads / num_kv_heads;
  const WsLayout w = ws_layout(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, pages_per_split);
  PKV_REQUIRE(workspace != nullptr && workspace_bytes >= w.total,
              "paged_decode: workspace of %lld bytes is smaller than the %lld bytes required",
              static_cast<long long>(workspace_bytes), static_cast<long long>(w.total));
  PKV_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "paged_decode: workspace must be 256-byte aligned");
  PKV_REQUIRE(w.max_units < (1ll << 31), "paged_decode: too many work units");
  const Workspace ws = carve(workspace, w);

  const float scale_log2 = scale * kLog2e;
  const uintptr_t align_bits = reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(key_pool) |
                               reinterpret_cast<uintptr_t>(value_pool);
  const int64_t rows = (num_pages - 1) * (sp / std::max<int64_t>(head_dim, 1)) +
                       (num_kv_heads - 1) * (sh / std::max<int64_t>(head_dim, 1)) + block_size;
  const bool tc_ok = !(flags & PKV_DECODE_CUDA_CORES) && (dtype == PKV_DTYPE_F16 || dtype == PKV_DTYPE_BF16) &&
                     (head_dim == 64 || head_dim == 128 || head_dim == 256) && block_size % 16 == 0 && group <= 8 &&
                     num_kv_heads <= 256 && ss == head_dim && sp % head_dim == 0 && sh % head_dim == 0 &&
                     (align_bits % 16) == 0 && (q_sb % 8) == 0 && (q_sh % 8) == 0 && rows < (1ll << 31) &&
                     sp / head_dim < (1ll << 31) && num_pages < (1ll << 31);
  if (tc_ok) {
    CUtensorMap km, vm;
    int st = encode_pool_map(&km, key_pool, dtype, head_dim, rows);
    if (st != PKV_OK) return st;
    st = encode_pool_map(&vm, value_pool, dtype, head_dim, rows);
    if (st != PKV_OK) return st;
    TcArgs<I> a{query, q_sb, q_sh, static_cast<const I*>(tables), table_stride, static_cast<int32_t>(max_blocks),
                static_cast<const I*>(seq_lens), static_cast<int32_t>(num_pages), static_cast<int32_t>(block_size),
                static_cast<int32_t>(sp / head_dim), static_cast<int32_t>(sh / head_dim),
                static_cast<int32_t>(num_kv_heads), static_cast<int32_t>(group), static_cast<int32_t>(batch),
                static_cast<int32_t>(pages_per_split), scale_log2, ws, output, o_sb, o_sh, error_flag};
    a.chained = (flags & PKV_DECODE_CHAINED) ? 1 : 0;
    a.prefetch = (flags & PKV_DECODE_PREFETCH) ? 1 : 0;
    bump_stat(kStatDecodeTensorCore);
    if (dtype == PKV_DTYPE_F16) {
      if (head_dim == 64) return launch_tc<__half, I, 64>(a, km, vm, stream);
      if (head_dim == 128) return launch_tc<__half, I, 128>(a, km, vm, stream);
      return launch_tc<__half, I, 256>(a, km, vm, stream);
    }
    if (head_dim == 64) return launch_tc<__nv_bfloat16, I, 64>(a, km, vm, stream);
    if (head_dim == 128) return launch_tc<__nv_bfloat16, I, 128>(a, km, vm, stream);
    return launch_tc<__nv_bfloat16, I, 256>(a, km, vm, stream);
  }
  PlanArgs<I> plan{static_cast<const I*>(seq_lens), -1, static_cast<int32_t>(batch), static_cast<int32_t>(num_kv_heads),
                   static_cast<int32_t>(num_q_heads), static_cast<int32_t>(block_size),
                   static_cast<int32_t>(max_blocks), static_cast<int32_t>(pages_per_split),
                   static_cast<int32_t>(pages_per_split_min(block_size)), ws, static_cast<char*>(output), o_sb * es,
                   o_sh * es, static_cast<int32_t>(head_dim * es), error_flag};
  decode_plan_kernel<I><<<1, 1024, 0, stream>>>(plan);
  int st = cuda_status(cudaGetLastError(), "decode_plan_kernel launch");
  if (st != PKV_OK) return st;
  GenArgs<I> g{query, q_sb, q_sh, key_pool, value_pool, nullptr, nullptr, nullptr, 0, num_pages, block_size, head_dim,
               sp, sh, ss, static_cast<const I*>(tables), table_stride, max_blocks, static_cast<const I*>(seq_lens),
               -1, static_cast<int32_t>(batch), static_cast<int32_t>(num_kv_heads), static_cast<int32_t>(group),
               scale_log2, ws, output, o_sb, o_sh, error_flag};
  bump_stat(kStatDecodeGeneric);
  const int64_t grid = std::min<int64_t>(w.max_units, static_cast<int64_t>(device_sms()) * 8);
  if (dtype == PKV_DTYPE_F32) return launch_generic<float, I>(g, std::max<int64_t>(grid, 1), stream);
  if (dtype == PKV_DTYPE_F16) return launch_generic<__half, I>(g, std::max<int64_t>(grid, 1), stream);
  return launch_generic<__nv_bfloat16, I>(g, std::max<int64_t>(grid, 1), stream);
}

template <typename I>
int run_decode_fp8(const void* query, int64_t q_sb, int64_t q_sh, const void* key_pool, const void* value_pool,
                   const float* k_scales, const float* v_scales, int64_t scale_sp, int64_t scale_sh,
                   int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim, int64_t sp,
                   int64_t sh, int64_t ss, const void* tables, int64_t table_stride, int64_t max_blocks,
                   const void* seq_lens, int64_t batch, int64_t num_q_heads, float scale, int64_t pages_per_split,
                   void* workspace, int64_t workspace_bytes, void* output, int64_t o_sb, int64_t o_sh, int dtype,
                   int flags, int32_t* error_flag, cudaStream_t stream) {
  const int64_t group = num_q_heads / num_kv_heads;
  const WsLayout w = ws_layout(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, pages_per_split);
  PKV_REQUIRE(workspace != nullptr && workspace_bytes >= w.total,
              "paged_decode_fp8: workspace of %lld bytes is smaller than the %lld bytes required",
              static_cast<long long>(workspace_bytes), static_cast<long long>(w.total));
  PKV_REQUIRE(reinterpret_cast<uintptr_t>(workspace) % 256 == 0, "paged_decode_fp8: workspace must be 256-byte aligned");
  const uintptr_t align_bits = reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(key_pool) |
                               reinterpret_cast<uintptr_t>(value_pool) | reinterpret_cast<uintptr_t>(k_scales) |
                               reinterpret_cast<uintptr_t>(v_scales);
  const int64_t rows = (num_pages - 1) * (sp / head_dim) + (num_kv_heads - 1) * (sh / head_dim) + block_size;
  PKV_UNSUPPORTED(dtype == PKV_DTYPE_F16 || dtype == PKV_DTYPE_BF16,
                  "paged_decode_fp8: query/output must be float16 or bfloat16");
  PKV_UNSUPPORTED(head_dim == 128 || head_dim == 256, "paged_decode_fp8: head_dim must be 128 or 256");
  PKV_UNSUPPORTED(block_size % 16 == 0 && group <= 8,
                  "paged_decode_fp8: block_size must be a multiple of 16 and at most 8 query heads share a KV head");
  PKV_REQUIRE(ss == head_dim && sp % head_dim == 0 && sh % head_dim == 0,
              "paged_decode_fp8: pool rows of head_dim bytes, one slot after another");
  PKV_REQUIRE(scale_sp % 4 == 0 && scale_sh % 4 == 0 && scale_sh >= block_size,
              "paged_decode_fp8: scale pools (pages, kv heads, block_size) with 16-byte aligned head rows");
  PKV_REQUIRE((align_bits % 16) == 0 && (q_sb % 8) == 0 && (q_sh % 8) == 0,
              "paged_decode_fp8: 16-byte aligned pools, scales and query rows");
  PKV_REQUIRE(rows < (1ll << 31) && num_pages < (1ll << 31), "paged_decode_fp8: pool too large");
  const Workspace ws = carve(workspace, w);
  CUtensorMap km, vm;
  int st = encode_pool_map_fp8(&km, key_pool, head_dim, rows);
  if (st != PKV_OK) return st;
  st = encode_pool_map_fp8(&vm, value_pool, head_dim, rows);
  if (st != PKV_OK) return st;
  TcArgs<I> a{query, q_sb, q_sh, static_cast<const I*>(tables), table_stride, static_cast<int32_t>(max_blocks),
              static_cast<const I*>(seq_lens), static_cast<int32_t>(num_pages), static_cast<int32_t>(block_size),
              static_cast<int32_t>(sp / head_dim), static_cast<int32_t>(sh / head_dim),
              static_cast<int32_t>(num_kv_heads), static_cast<int32_t>(group), static_cast<int32_t>(batch),
              static_cast<int32_t>(pages_per_split), scale * kLog2e, ws, output, o_sb, o_sh, error_flag,
              k_scales, v_scales, scale_sp, scale_sh};
  a.chained = (flags & PKV_DECODE_CHAINED) ? 1 : 0;
  a.prefetch = (flags & PKV_DECODE_PREFETCH) ? 1 : 0;
  bump_stat(kStatDecodeFp8);
  if (dtype == PKV_DTYPE_F16) {
    if (head_dim == 128) return launch_tc<__half, I, 128, true>(a, km, vm, stream);
    return launch_tc<__half, I, 256, true>(a, km, vm, stream);
  }
  if (head_dim == 128) return launch_tc<__nv_bfloat16, I, 128, true>(a, km, vm, stream);
  return launch_tc<__nv_bfloat16, I, 256, true>(a, km, vm, stream);
}

}  // namespace
}  // namespace pkv

using namespace pkv;

namespace pkv {
namespace {

// Upper bound of ws_layout(...).total in floating point, so that sizes whose exact layout would overflow
// int64 are rejected before the layout is computed.
double workspace_estimate(int64_t batch, int64_t num_q_heads, int64_t num_kv_heads, int64_t head_dim,
                          int64_t max_blocks, int64_t block_size, int64_t pages_per_split) {
  const double bh = static_cast<double>(batch) * static_cast<double>(num_kv_heads);
  const double pps = static_cast<double>(pages_per_split > 0 ? pages_per_split : pages_per_split_min(block_size));
  double units = bh * std::ceil(static_cast<double>(std::max<int64_t>(max_blocks, 1)) / pps);
  if (pages_per_split <= 0) units = std::min(units, static_cast<double>(kTargetUnits) + bh);
  const double slots = std::max(units, 2.0 * kMaxStreamWarps);
  const double group = static_cast<double>(num_q_heads / num_kv_heads);
  return 1024.0 + bh * 4.0 + units * 16.0 + slots * group * (8.0 + 4.0 * static_cast<double>(head_dim));
}

// Host-side checks of pkv_paged_decode's arguments (every size and pointer the launch and the workspace
// layout depend on). Null pointers are accepted for an empty batch, which launches nothing; with
// `sizes_only` the pointers and the scale are not checked.
int check_decode_args(const void* query, const void* key_pool, const void* value_pool, int64_t num_pages,
                      int64_t num_kv_heads, int64_t block_size, int64_t head_dim, const void* block_tables,
                      int64_t max_blocks, const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                      float scale, int64_t pages_per_split, const void* output, int dtype, bool sizes_only = false) {
  PKV_REQUIRE(dtype_size(dtype) > 0, "paged_decode: unsupported dtype %d", dtype);
  PKV_REQUIRE(index_dtype == PKV_INDEX_I32 || index_dtype == PKV_INDEX_I64, "paged_decode: bad index dtype");
  PKV_REQUIRE(batch >= 0 && batch < (1 << 30), "paged_decode: batch out of range");
  PKV_REQUIRE(num_kv_heads > 0 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0,
              "paged_decode: num_q_heads (%lld) must be a positive multiple of num_kv_heads (%lld)",
              static_cast<long long>(num_q_heads), static_cast<long long>(num_kv_heads));
  PKV_REQUIRE(num_kv_heads <= 256, "paged_decode: at most 256 KV heads");
  PKV_REQUIRE(head_dim > 0 && head_dim <= 1024, "paged_decode: head_dim must be in [1, 1024]");
  PKV_REQUIRE(block_size > 0 && num_pages > 0 && max_blocks > 0 && max_blocks < (1 << 30),
              "paged_decode: block_size, num_pages and max_blocks must be positive");
  PKV_REQUIRE(workspace_estimate(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, pages_per_split) <
                  0x1p60,
              "paged_decode: the workspace of this call would exceed 2^60 bytes");
  if (batch == 0 || sizes_only) return PKV_OK;
  PKV_REQUIRE(query && key_pool && value_pool && block_tables && seq_lens && output,
              "paged_decode: null pointer argument");
  PKV_REQUIRE(std::isfinite(scale), "paged_decode: scale must be finite");
  return PKV_OK;
}

}  // namespace
}  // namespace pkv

extern "C" int pkv_paged_decode_fp8_ex(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                                       const void* key_pool, const void* value_pool, const float* key_scales,
                                       const float* value_scales, int64_t scale_stride_page,
                                       int64_t scale_stride_head, int64_t num_pages, int64_t num_kv_heads,
                                       int64_t block_size, int64_t head_dim, int64_t stride_page, int64_t stride_head,
                                       int64_t stride_slot, const void* block_tables, int64_t table_stride,
                                       int64_t max_blocks, const void* seq_lens, int index_dtype, int64_t batch,
                                       int64_t num_q_heads, float scale, int64_t pages_per_split, void* workspace,
                                       int64_t workspace_bytes, void* output, int64_t o_stride_batch,
                                       int64_t o_stride_head, int dtype, int flags, int32_t* error_flag,
                                       void* stream) {
  clear_error();
  PKV_REQUIRE((flags & ~(PKV_DECODE_CHAINED | PKV_DECODE_PREFETCH)) == 0, "paged_decode_fp8: unknown flags 0x%x",
              flags);
  PKV_REQUIRE(!(flags & PKV_DECODE_PREFETCH) || (flags & PKV_DECODE_CHAINED),
              "paged_decode_fp8: PKV_DECODE_PREFETCH needs PKV_DECODE_CHAINED");
  PKV_REQUIRE(dtype_size(dtype) > 0, "paged_decode_fp8: unsupported dtype %d", dtype);
  PKV_REQUIRE(index_dtype == PKV_INDEX_I32 || index_dtype == PKV_INDEX_I64, "paged_decode_fp8: bad index dtype");
  PKV_REQUIRE(batch >= 0 && batch < (1 << 30), "paged_decode_fp8: batch out of range");
  PKV_REQUIRE(num_kv_heads > 0 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0 && num_kv_heads <= 256,
              "paged_decode_fp8: num_q_heads must be a positive multiple of num_kv_heads (<= 256)");
  PKV_REQUIRE(block_size > 0 && num_pages > 0 && max_blocks > 0 && max_blocks < (1 << 30),
              "paged_decode_fp8: block_size, num_pages and max_blocks must be positive");
  if (batch == 0) return PKV_OK;
  PKV_REQUIRE(query && key_pool && value_pool && key_scales && value_scales && block_tables && seq_lens && output,
              "paged_decode_fp8: null pointer argument");
  PKV_REQUIRE(std::isfinite(scale), "paged_decode_fp8: scale must be finite");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (index_dtype == PKV_INDEX_I32)
    return run_decode_fp8<int32_t>(query, q_stride_batch, q_stride_head, key_pool, value_pool, key_scales,
                                   value_scales, scale_stride_page, scale_stride_head, num_pages, num_kv_heads,
                                   block_size, head_dim, stride_page, stride_head, stride_slot, block_tables,
                                   table_stride, max_blocks, seq_lens, batch, num_q_heads, scale, pages_per_split,
                                   workspace, workspace_bytes, output, o_stride_batch, o_stride_head, dtype,
                                   flags, error_flag, s);
  return run_decode_fp8<int64_t>(query, q_stride_batch, q_stride_head, key_pool, value_pool, key_scales,
                                 value_scales, scale_stride_page, scale_stride_head, num_pages, num_kv_heads,
                                 block_size, head_dim, stride_page, stride_head, stride_slot, block_tables,
                                 table_stride, max_blocks, seq_lens, batch, num_q_heads, scale, pages_per_split,
                                 workspace, workspace_bytes, output, o_stride_batch, o_stride_head, dtype, flags,
                                 error_flag, s);
}

extern "C" int pkv_paged_decode_fp8(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                                    const void* key_pool, const void* value_pool, const float* key_scales,
                                    const float* value_scales, int64_t scale_stride_page, int64_t scale_stride_head,
                                    int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                                    int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                                    const void* block_tables, int64_t table_stride, int64_t max_blocks,
                                    const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                                    float scale, int64_t pages_per_split, void* workspace, int64_t workspace_bytes,
                                    void* output, int64_t o_stride_batch, int64_t o_stride_head, int dtype,
                                    int32_t* error_flag, void* stream) {
  return pkv_paged_decode_fp8_ex(query, q_stride_batch, q_stride_head, key_pool, value_pool, key_scales,
                                 value_scales, scale_stride_page, scale_stride_head, num_pages, num_kv_heads,
                                 block_size, head_dim, stride_page, stride_head, stride_slot, block_tables,
                                 table_stride, max_blocks, seq_lens, index_dtype, batch, num_q_heads, scale,
                                 pages_per_split, workspace, workspace_bytes, output, o_stride_batch, o_stride_head,
                                 dtype, 0, error_flag, stream);
}

extern "C" int64_t pkv_paged_decode_workspace_size(int64_t batch, int64_t num_q_heads, int64_t num_kv_heads,
                                                   int64_t head_dim, int64_t max_blocks, int64_t block_size,
                                                   int64_t pages_per_split) {
  if (batch < 0 || num_kv_heads <= 0 || num_q_heads <= 0 || head_dim <= 0 || block_size <= 0) return -1;
  if (max_blocks < 0 || max_blocks >= (1 << 30) || num_kv_heads > 256) return -1;
  if (workspace_estimate(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, pages_per_split) >=
      0x1p60)
    return -1;
  return ws_layout(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, pages_per_split).total;
}

extern "C" int pkv_paged_decode_ex(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                                   const void* key_pool, const void* value_pool, int64_t num_pages,
                                   int64_t num_kv_heads, int64_t block_size, int64_t head_dim, int64_t stride_page,
                                   int64_t stride_head, int64_t stride_slot, const void* block_tables,
                                   int64_t table_stride, int64_t max_blocks, const void* seq_lens, int index_dtype,
                                   int64_t batch, int64_t num_q_heads, float scale, int64_t pages_per_split,
                                   void* workspace, int64_t workspace_bytes, void* output, int64_t o_stride_batch,
                                   int64_t o_stride_head, int dtype, int flags, int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE((flags & ~(PKV_DECODE_CHAINED | PKV_DECODE_CUDA_CORES | PKV_DECODE_PREFETCH)) == 0,
              "paged_decode: unknown flags 0x%x", flags);
  PKV_REQUIRE(!(flags & PKV_DECODE_PREFETCH) || (flags & PKV_DECODE_CHAINED),
              "paged_decode: PKV_DECODE_PREFETCH needs PKV_DECODE_CHAINED");
  const int st = check_decode_args(query, key_pool, value_pool, num_pages, num_kv_heads, block_size, head_dim,
                                   block_tables, max_blocks, seq_lens, index_dtype, batch, num_q_heads, scale,
                                   pages_per_split, output, dtype);
  if (st != PKV_OK) return st;
  if (batch == 0) return PKV_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (index_dtype == PKV_INDEX_I32) {
    return run_decode<int32_t>(query, q_stride_batch, q_stride_head, key_pool, value_pool, num_pages, num_kv_heads,
                               block_size, head_dim, stride_page, stride_head, stride_slot, block_tables, table_stride,
                               max_blocks, seq_lens, batch, num_q_heads, scale, pages_per_split, workspace,
                               workspace_bytes, output, o_stride_batch, o_stride_head, dtype, flags, error_flag, s);
  }
  return run_decode<int64_t>(query, q_stride_batch, q_stride_head, key_pool, value_pool, num_pages, num_kv_heads,
                             block_size, head_dim, stride_page, stride_head, stride_slot, block_tables, table_stride,
                             max_blocks, seq_lens, batch, num_q_heads, scale, pages_per_split, workspace,
                             workspace_bytes, output, o_stride_batch, o_stride_head, dtype, flags, error_flag, s);
}

extern "C" int pkv_paged_decode(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                                const void* key_pool, const void* value_pool, int64_t num_pages, int64_t num_kv_heads,
                                int64_t block_size, int64_t head_dim, int64_t stride_page, int64_t stride_head,
                                int64_t stride_slot, const void* block_tables, int64_t table_stride,
                                int64_t max_blocks, const void* seq_lens, int index_dtype, int64_t batch,
                                int64_t num_q_heads, float scale, int64_t pages_per_split, void* workspace,
                                int64_t workspace_bytes, void* output, int64_t o_stride_batch, int64_t o_stride_head,
                                int dtype, int32_t* error_flag, void* stream) {
  return pkv_paged_decode_ex(query, q_stride_batch, q_stride_head, key_pool, value_pool, num_pages, num_kv_heads,
                             block_size, head_dim, stride_page, stride_head, stride_slot, block_tables, table_stride,
                             max_blocks, seq_lens, index_dtype, batch, num_q_heads, scale, pages_per_split, workspace,
                             workspace_bytes, output, o_stride_batch, o_stride_head, dtype, 0, error_flag, stream);
}

// ---- decode with library-owned scratch --------------------------------------------------------------------
// Some callers cannot allocate device memory at all: a serving runtime that reserved nearly all HBM
// for its KV page pools up front and forbids later allocations, or a host reached through an FFI
// (cgo, JNI) that hands this library raw pointers of buffers it already owns and has no device
// allocator to call. For them pkv_paged_decode_static_scratch runs the same decode with its scratch
// in the file-scope array below instead of a caller workspace. The array is PKV_DECODE_STATIC_SCRATCH_BYTES
// (32 MiB) per GPU, is held on every GPU that loads this library until the process exits, and is
// shared by every call on that GPU: two calls that overlap on the GPU (different streams, no ordering)
// race on it. Its device address is looked up once per device and cached for the life of the process,
// so the entry point must not be used after a cudaDeviceReset (or any reset of the primary context)
// in the same process: the module is reloaded then and the cached address is stale.
static __device__ __align__(256) unsigned char g_decode_static_scratch[PKV_DECODE_STATIC_SCRATCH_BYTES];

namespace pkv {
namespace {

constexpr int kMaxDevices = 64;
std::mutex g_static_scratch_mutex;
void* g_static_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device, looked up once per device. In host code
// the array's name is only a host-side stand-in, so kernels must be given this address instead.
int static_scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e, "paged_decode_static_scratch: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDevices) {
    set_error("paged_decode_static_scratch: device %d beyond the %d supported", dev, kMaxDevices);
    return PKV_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_static_scratch_mutex);
  if (g_static_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_decode_static_scratch);
    if (e != cudaSuccess) return cuda_status(e, "paged_decode_static_scratch: cudaGetSymbolAddress");
    g_static_scratch_ptr[dev] = ptr;
  }
  *out = g_static_scratch_ptr[dev];
  return PKV_OK;
}

}  // namespace
}  // namespace pkv

extern "C" int pkv_paged_decode_static_scratch(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                                               const void* key_pool, const void* value_pool, int64_t num_pages,
                                               int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                                               int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                                               const void* block_tables, int64_t table_stride, int64_t max_blocks,
                                               const void* seq_lens, int index_dtype, int64_t batch,
                                               int64_t num_q_heads, float scale, int64_t pages_per_split,
                                               void* output, int64_t o_stride_batch, int64_t o_stride_head,
                                               int dtype, int32_t* error_flag, void* stream) {
  clear_error();
  // Every argument is checked before anything is enqueued: a rejected call leaves the shared array as
  // it was, and the layout below is only computed from sizes whose products cannot overflow.
  int st = check_decode_args(query, key_pool, value_pool, num_pages, num_kv_heads, block_size, head_dim,
                             block_tables, max_blocks, seq_lens, index_dtype, batch, num_q_heads, scale,
                             pages_per_split, output, dtype, /*sizes_only=*/true);
  if (st != PKV_OK) return st;
  const WsLayout w = ws_layout(batch, num_q_heads, num_kv_heads, head_dim, max_blocks, block_size, pages_per_split);
  PKV_REQUIRE(w.total <= PKV_DECODE_STATIC_SCRATCH_BYTES && w.units_off <= w.total,
              "paged_decode_static_scratch: this call needs %lld bytes of scratch but the static scratch holds "
              "%lld bytes; use pkv_paged_decode with a caller workspace",
              static_cast<long long>(w.total), static_cast<long long>(PKV_DECODE_STATIC_SCRATCH_BYTES));
  st = check_decode_args(query, key_pool, value_pool, num_pages, num_kv_heads, block_size, head_dim, block_tables,
                         max_blocks, seq_lens, index_dtype, batch, num_q_heads, scale, pages_per_split, output, dtype);
  if (st != PKV_OK) return st;
  if (batch == 0) return PKV_OK;
  void* scratch = nullptr;
  st = static_scratch_address(&scratch);
  if (st != PKV_OK) return st;
  // The counters and the plan header keep the previous call's values; the decode expects them zero.
  st = cuda_status(cudaMemsetAsync(scratch, 0, static_cast<size_t>(w.units_off), static_cast<cudaStream_t>(stream)),
                   "paged_decode_static_scratch: clearing the counters");
  if (st != PKV_OK) return st;
  return pkv_paged_decode(query, q_stride_batch, q_stride_head, key_pool, value_pool, num_pages, num_kv_heads,
                          block_size, head_dim, stride_page, stride_head, stride_slot, block_tables, table_stride,
                          max_blocks, seq_lens, index_dtype, batch, num_q_heads, scale, pages_per_split, scratch,
                          PKV_DECODE_STATIC_SCRATCH_BYTES, output, o_stride_batch, o_stride_head, dtype,
                          error_flag, stream);
}

extern "C" int pkv_lse_merge(const float* partial_out, const float* partial_lse, int64_t num_parts, int64_t rows,
                             int64_t head_dim, void* out, int64_t out_stride_row, float* out_lse, int dtype,
                             void* stream) {
  clear_error();
  PKV_REQUIRE(dtype_size(dtype) > 0, "lse_merge: unsupported dtype %d", dtype);
  PKV_REQUIRE(num_parts > 0 && rows >= 0 && head_dim > 0, "lse_merge: bad sizes");
  if (rows == 0) return PKV_OK;
  PKV_REQUIRE(partial_out && partial_lse && out, "lse_merge: null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (dtype == PKV_DTYPE_F32)
    lse_merge_kernel<float><<<rows, 256, 0, s>>>(partial_out, partial_lse, num_parts, rows, head_dim,
                                                 static_cast<float*>(out), out_stride_row, out_lse);
  else if (dtype == PKV_DTYPE_F16)
    lse_merge_kernel<__half><<<rows, 256, 0, s>>>(partial_out, partial_lse, num_parts, rows, head_dim,
                                                  static_cast<__half*>(out), out_stride_row, out_lse);
  else
    lse_merge_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>(partial_out, partial_lse, num_parts, rows, head_dim,
                                                         static_cast<__nv_bfloat16*>(out), out_stride_row, out_lse);
  bump_stat(kStatLseMerge);
  return cuda_status(cudaGetLastError(), "lse_merge launch");
}

extern "C" int pkv_paged_attention_decode(const void* query, const int64_t* block_table, int64_t table_len,
                                          const void* key_blocks, const void* value_blocks, int64_t batch,
                                          int64_t heads, int64_t physical_blocks, int64_t block_size,
                                          int64_t head_dim, int64_t sequence_length, void* output, int dtype,
                                          int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE(dtype_size(dtype) > 0, "paged_attention_decode: unsupported dtype %d", dtype);
  PKV_REQUIRE(sequence_length > 0, "sequence_length must be positive");
  PKV_REQUIRE(block_size > 0, "block_size must be positive");
  PKV_REQUIRE(batch > 0 && batch <= INT32_MAX, "batch must be positive and fit int32");
  PKV_REQUIRE(heads > 0 && heads <= 256, "heads must be in [1, 256]");
  PKV_REQUIRE(head_dim > 0 && head_dim <= 1024, "head_dim must be in [1, 1024]");
  PKV_REQUIRE(physical_blocks > 0 && physical_blocks <= INT32_MAX,
              "physical block count must be positive and fit int32");
  PKV_REQUIRE(table_len >= ceil_div(sequence_length, block_size), "block_table does not cover sequence_length");
  PKV_REQUIRE(query && block_table && key_blocks && value_blocks && output, "paged_attention_decode: null pointer");
  GenArgs<int64_t> g{query, heads * head_dim, head_dim, key_blocks, value_blocks, nullptr, nullptr, nullptr,
                     heads * physical_blocks * block_size * head_dim, physical_blocks, block_size, head_dim,
                     block_size * head_dim, physical_blocks * block_size * head_dim, head_dim, block_table, 0,
                     table_len, nullptr, sequence_length, static_cast<int32_t>(batch), static_cast<int32_t>(heads), 1,
                     kLog2e / std::sqrt(static_cast<float>(head_dim)), Workspace{}, output, heads * head_dim,
                     head_dim, error_flag};
  bump_stat(kStatRefSingle);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t grid = batch * heads;
  if (dtype == PKV_DTYPE_F32) return launch_generic<float, int64_t>(g, grid, s);
  if (dtype == PKV_DTYPE_F16) return launch_generic<__half, int64_t>(g, grid, s);
  return launch_generic<__nv_bfloat16, int64_t>(g, grid, s);
}

extern "C" int pkv_paged_attention_decode_batched(const void* query, const int64_t* block_tables, int64_t max_blocks,
                                                  const void* const* key_block_ptrs,
                                                  const void* const* value_block_ptrs,
                                                  const int64_t* physical_block_counts,
                                                  const int64_t* sequence_lengths, int64_t batch, int64_t heads,
                                                  int64_t block_size, int64_t head_dim, void* output, int dtype,
                                                  int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE(dtype_size(dtype) > 0, "paged_attention_decode_batched: unsupported dtype %d", dtype);
  PKV_REQUIRE(block_size > 0, "block_size must be positive");
  PKV_REQUIRE(batch > 0 && batch <= INT32_MAX, "batch must be positive and fit int32");
  PKV_REQUIRE(heads > 0 && heads <= 256, "heads must be in [1, 256]");
  PKV_REQUIRE(head_dim > 0 && head_dim <= 1024, "head_dim must be in [1, 1024]");
  PKV_REQUIRE(max_blocks > 0 && max_blocks <= INT32_MAX, "max_blocks must be positive and fit int32");
  PKV_REQUIRE(query && block_tables && key_block_ptrs && value_block_ptrs && physical_block_counts &&
                  sequence_lengths && output,
              "paged_attention_decode_batched: null pointer");
  GenArgs<int64_t> g{query, heads * head_dim, head_dim, nullptr, nullptr, key_block_ptrs, value_block_ptrs,
                     physical_block_counts, 0, 0, block_size, head_dim, block_size * head_dim, 0, head_dim,
                     block_tables, max_blocks, max_blocks, sequence_lengths, -1, static_cast<int32_t>(batch),
                     static_cast<int32_t>(heads), 1, kLog2e / std::sqrt(static_cast<float>(head_dim)), Workspace{},
                     output, heads * head_dim, head_dim, error_flag};
  bump_stat(kStatRefBatched);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t grid = batch * heads;
  if (dtype == PKV_DTYPE_F32) return launch_generic<float, int64_t>(g, grid, s);
  if (dtype == PKV_DTYPE_F16) return launch_generic<__half, int64_t>(g, grid, s);
  return launch_generic<__nv_bfloat16, int64_t>(g, grid, s);
}

extern "C" int pkv_paged_decode_request_pools(const void* query, int64_t q_stride_batch, int64_t q_stride_head,
                                              const void* const* key_pool_ptrs, const void* const* value_pool_ptrs,
                                              const int64_t* pool_pages, int64_t num_kv_heads, int64_t block_size,
                                              int64_t head_dim, const int64_t* block_tables, int64_t max_blocks,
                                              const int64_t* seq_lens, int64_t batch, int64_t num_q_heads,
                                              float scale, void* output, int64_t o_stride_batch,
                                              int64_t o_stride_head, int dtype, int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE(dtype_size(dtype) > 0, "paged_decode_request_pools: unsupported dtype %d", dtype);
  PKV_REQUIRE(batch >= 0 && batch <= INT32_MAX, "paged_decode_request_pools: batch out of range");
  PKV_REQUIRE(num_kv_heads > 0 && num_kv_heads <= 256 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0,
              "paged_decode_request_pools: num_q_heads must be a positive multiple of num_kv_heads (<= 256)");
  PKV_REQUIRE(head_dim > 0 && head_dim <= 1024, "paged_decode_request_pools: head_dim must be in [1, 1024]");
  PKV_REQUIRE(block_size > 0 && max_blocks > 0 && max_blocks <= INT32_MAX,
              "paged_decode_request_pools: block_size and max_blocks must be positive");
  PKV_REQUIRE(std::isfinite(scale), "paged_decode_request_pools: scale must be finite");
  if (batch == 0) return PKV_OK;
  PKV_REQUIRE(query && key_pool_ptrs && value_pool_ptrs && pool_pages && block_tables && seq_lens && output,
              "paged_decode_request_pools: null pointer argument");
  const int64_t group = num_q_heads / num_kv_heads;
  GenArgs<int64_t> g{query, q_stride_batch, q_stride_head, nullptr, nullptr, key_pool_ptrs, value_pool_ptrs,
                     pool_pages, 0, 0, block_size, head_dim, num_kv_heads * block_size * head_dim,
                     block_size * head_dim, head_dim, block_tables, max_blocks, max_blocks, seq_lens, -1,
                     static_cast<int32_t>(batch), static_cast<int32_t>(num_kv_heads), static_cast<int32_t>(group),
                     scale * kLog2e, Workspace{}, output, o_stride_batch, o_stride_head, error_flag};
  bump_stat(kStatRefBatched);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t grid = batch * num_kv_heads;
  if (dtype == PKV_DTYPE_F32) return launch_generic<float, int64_t>(g, grid, s);
  if (dtype == PKV_DTYPE_F16) return launch_generic<__half, int64_t>(g, grid, s);
  return launch_generic<__nv_bfloat16, int64_t>(g, grid, s);
}
