// Attention output stage of a full-attention layer, fused with its tensor-parallel all-reduce:
//
//   x        = heads * sigmoid(gate)                                  (torch's rounding points)
//   partial  = (x @ dequant(W_local)^T).to(out dtype)                 (e4m3 W, bf16 128x128 block scales)
//   out      = sum over TP ranks of partial                           (fixed rank order, fp32, one rounding)
//
// restating src/tp_runtime.py:672-695 (_tp_full_attention_finish_from_heads), the linear of
// src/reference_ops.py:436-506 and the NCCL SUM of TpRuntime.all_reduce_sum (src/tp_runtime.py:288-298).
//
// Three launches, chained by programmatic dependent launch so that each starts while its
// predecessor drains:
//   1. oproj_gate_kernel: x once per element, written as f16 rows (tokens, K_local) to the workspace;
//      it also clears the fp32 split-k sums and tile counters of the projection.
//   2. oproj_kernel: KS CTAs along K per tile. A CTA owns 128 hidden rows (one scale block) x TN
//      tokens (32, 64 or 128) x K_local / KS. A producer warp streams its e4m3 weight tiles and f16 x
//      tiles in by TMA (the weight loads are issued before the wait on kernel 1); converter warps widen
//      the weight to f16 straight into tensor memory (the A operand, four buffers); one thread issues
//      tcgen05.mma 128 x TN x 16 against the x tile in shared memory (the B operand), one TMEM
//      accumulator per 128-k block (two buffers), which reader warps read back and add with the block's
//      scale in registers (exact per-block scaling, fp32). With KS > 1 the partial tiles meet in an
//      fp32 sum in the workspace (vector float reductions) and the last CTA of a tile to arrive (atomic
//      counter, nobody waits) finishes the tile; with KS = 1 the CTA finishes its own. Finishing rounds
//      the sum to the output dtype and either stores it (one rank) or stores it into its own and every
//      peer's exchange buffer over NVLink (plain stores to IPC-mapped peer memory) as 8-byte words that
//      carry the call's epoch next to the data. This kernel never waits on another CTA or GPU.
//   3. oproj_finish_kernel (TP > 1): per slice, reads every rank's words of the slice, each until it
//      carries this call's epoch (bounded), sums the TP partials in rank order and writes the output.
// A word is stored and loaded as one 64-bit access, so its epoch proves its data: no flag, no fence,
// no release on the pushing side (a system-scope fence or release per call costs microseconds). The
// exchange buffers are double-buffered by call parity and the epoch is kept in device memory, so the
// step can be captured in a CUDA graph: a rank cannot reuse a buffer before every peer finished reading
// it, since it needs their words of the next call first, which a peer writes only after its finishing
// kernel of this call has completed.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstring>
#include <mutex>
#include <type_traits>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr int kOpIssueWarp = 12;              // MMA issuer, TMEM owner (after the converter and reader warps)
constexpr int kOpProdWarp = 13;               // TMA producer, barrier owner
constexpr int kOpThreads = 32 * (kOpProdWarp + 1);
constexpr int kOpABufs = 4;                   // A (widened weight) buffers in TMEM, 64 columns each
constexpr int kOpRows = 128;                  // hidden rows per CTA = one scale block = the MMA's M
constexpr int kOpWBytes = kOpRows * 128;      // e4m3 weight tile of one 128-k block
constexpr int kOpPitch = kOpRows + 4;         // floats per token row of the partial tile (bank spread)
constexpr int kOpMinTokens = 32;              // the smaller token tile (sizes the tile counters)
constexpr float kLoScale = 2048.f;            // the lo part of fp32 activations is stored times 2^11
constexpr int kOpMaxWorld = 8;
constexpr int kOpMaxSplit = 8;                // CTAs per tile along k
constexpr int kFinishSlices = 8;              // finishing CTAs per tile (row-quad slices)
constexpr uint64_t kOpWaitNs = 2000000000ull;  // bounded waits: 2 s
constexpr int64_t kCommHeader = 256;          // epoch, finished-CTA count; the data words follow

// XP = planes of x: 1 when the activations are 16-bit (exact in f16), 2 when they are fp32 and travel
// as hi = f16(x) plus lo = f16((x - hi) * 2^11), together within 2^-22 of x. TN = tokens per CTA (the
// MMA's N: 32, 64, or 128 with one plane). The partial tile of the split-k sum reuses the stage memory
// once every stage is consumed.
//
// Warp roles: kConvWarps converter warps (warp % 4 = the 32 TMEM lanes = weight rows they widen, warp / 4
// = the part of each 128-byte row), kReadWarps reader warps (warp % 4 = lanes, (warp - kConvWarps) / 4 =
// which kReadCols token columns of the accumulator they read and keep), the MMA issuer, the producer.
template <int XP, int TN>
struct OpCfg {
  static constexpr int kConvWarps = XP * TN >= 128 ? 4 : 8;
  static constexpr int kReadWarps = XP * TN >= 128 ? 8 : 4;
  static constexpr int kReadCols = TN * 4 / kReadWarps;  // token columns per reader thread (its registers)
  static constexpr int kConvUnits = 8 * 4 / kConvWarps;  // 16-byte units of a weight row per converter thread
  static_assert(kConvWarps + kReadWarps == kOpIssueWarp, "warp roles");
  static constexpr int kXBytes = TN * 256;         // f16 x tile of one 128-k block: two 64-k halves of TN rows
  static constexpr int kStageBytes = kOpWBytes + XP * kXBytes;
  // 128-k stages in flight per CTA: as many as 192 KB hold (one CTA per SM either way), so that a CTA's
  // whole k slice is usually in flight after one DRAM round trip
  static constexpr int kStages = (192 * 1024) / kStageBytes < 8 ? (192 * 1024) / kStageBytes : 8;
  static constexpr int kTileBytes = TN * kOpPitch * 4;
  static constexpr int kMaxBlocks = 256;           // 128-k blocks per CTA (their scales are preloaded)
  static constexpr int kBars = 2 * kStages + 2 * kOpABufs + 5;
  static constexpr int kSmem = 1024 + kStages * kStageBytes + kBars * 8 + 16 + kMaxBlocks * 4;
  static constexpr int kDCols = XP * TN;           // one block's accumulators (hi, lo planes)
  static constexpr int kTmemCols = 512;            // A x4 in [0, 256), D x2 from 256
  static_assert(kOpABufs * 64 + 2 * kDCols <= kTmemCols, "TMEM budget");
  static_assert(kReadCols % 32 == 0 && kReadCols <= 64, "reader registers");
  static_assert(kOpWBytes % 1024 == 0 && kXBytes % 1024 == 0 && (kXBytes / 2) % 1024 == 0,
                "TMA tiles stay 1024-byte aligned");
  static_assert(kStages * kStageBytes >= kTileBytes, "the partial tile fits in the stage memory");
};

struct GateArgs {
  const void* heads;
  int64_t h_sb, h_sh, h_ss;  // elements: batch, head, sequence strides (head_dim contiguous)
  const void* gate;
  int64_t g_sb, g_ss;        // elements: batch, sequence strides (K contiguous)
  int32_t seq_len, head_dim, k;
  int32_t hd_shift;          // log2(head_dim) when it is a power of two, else -1
  int64_t tokens;
  __half* x;                 // (tokens, k) f16 hi plane, followed by the lo plane when there is one
  int64_t plane;             // elements per plane
  float4* clear;             // the projection's split-k sums and tile counters, cleared every call
  int64_t clear_vec4;
};

// torch's result dtype of heads * sigmoid(gate): the common type, or float32 for mixed types.
template <typename A, typename B> struct Promote { using type = float; };
template <typename A> struct Promote<A, A> { using type = A; };

template <typename T>
__device__ __forceinline__ void load8(const T* p, float (&v)[8]) {
  if constexpr (std::is_same<T, float>::value) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const uint4 a = *reinterpret_cast<const uint4*>(p);
    const uint32_t w[4] = {a.x, a.y, a.z, a.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = unpack2<T>(w[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ float round_as(float v) {
  return Elem<T>::to_f(Elem<T>::from_f(v));
}

// The 8 consecutive k starting at k8 (head `head`, element d of it) of token m.
template <typename TH, typename TG, int XP>
__device__ __forceinline__ void gate_group(const GateArgs& a, int64_t m, int head, int d, int k8) {
  using TP = typename Promote<TH, TG>::type;
  const int64_t b = a.seq_len == 1 ? m : m / a.seq_len, s = m - b * a.seq_len;
  float h[8], g[8];
  load8(static_cast<const TH*>(a.heads) + b * a.h_sb + head * a.h_sh + s * a.h_ss + d, h);
  load8(static_cast<const TG*>(a.gate) + b * a.g_sb + s * a.g_ss + k8, g);
  uint32_t hi[4], lo[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float r[2];
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const float sig = round_as<TG>(1.f / (1.f + expf(-g[2 * j + e])));  // sigmoid in fp32, rounded to the gate's type
      r[e] = round_as<TP>(h[2 * j + e] * sig);                            // product rounded to the promoted type
    }
    hi[j] = pack2<__half>(r[0], r[1]);  // the tensor-core operand type
    if constexpr (XP == 2) {
      const float2 hf = unpack2<__half>(hi[j]);
      lo[j] = pack2<__half>((r[0] - hf.x) * kLoScale, (r[1] - hf.y) * kLoScale);
    }
  }
  __half* dst = a.x + m * a.k + k8;
  *reinterpret_cast<uint4*>(dst) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
  if constexpr (XP == 2) *reinterpret_cast<uint4*>(dst + a.plane) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
}

// Grid (ceil(k / 8 / 256), min(tokens, 65535)): thread x of block (bx, by) gates the 8 consecutive k
// starting at 8 (256 bx + x) of tokens by, by + gridDim.y, ... (no index divisions but the head's).
template <typename TH, typename TG, int XP>
__global__ void __launch_bounds__(256) oproj_gate_kernel(const GateArgs a) {
  using TP = typename Promote<TH, TG>::type;
  pdl_launch_dependents();
  pdl_wait();  // the heads come from the kernel before (a no-op unless launched chained)
  const int64_t lin = (static_cast<int64_t>(blockIdx.y) * gridDim.x + blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t all = static_cast<int64_t>(gridDim.x) * gridDim.y * blockDim.x;
  for (int64_t z = lin; z < a.clear_vec4; z += all) a.clear[z] = make_float4(0.f, 0.f, 0.f, 0.f);
  const int j8 = blockIdx.x * blockDim.x + threadIdx.x;
  if (j8 >= (a.k >> 3)) return;
  const int k8 = j8 * 8;
  const int head = a.hd_shift >= 0 ? k8 >> a.hd_shift : k8 / a.head_dim, d = k8 - head * a.head_dim;
  for (int64_t m = blockIdx.y; m < a.tokens; m += gridDim.y) {
    gate_group<TH, TG, XP>(a, m, head, d, k8);
  }
}
struct OpArgs {
  const __nv_bfloat16* scale;  // (hidden / 128, k / 128) bf16
  int64_t s_sn, s_sk;          // elements
  int32_t tokens, hidden, k;
  int32_t split, blocks;       // CTAs per cluster along k, 128-k blocks per CTA
  int32_t tn;                  // tokens per CTA
  void* out;
  int64_t o_st;                // elements per token row
  int32_t world, rank;
  char* bufs[kOpMaxWorld];     // exchange buffers (bufs[rank] local, the others IPC-mapped peers)
  int64_t capacity;            // tokens per exchange slot
  int64_t data_off;            // bytes from a buffer's start to its data slots
  int32_t* error_flag;
  float* sums;                 // (tokens, hidden) fp32 split-k sums, cleared by the gate kernel
  uint32_t* counters;          // per tile: CTAs of the tile that added their partial
};

__device__ __forceinline__ uint32_t* comm_state(const OpArgs& a) { return reinterpret_cast<uint32_t*>(a.bufs[a.rank]); }

// Exchange words: {bits of two 16-bit values (one fp32 value), call epoch} in one 64-bit word.
template <typename TO> constexpr int kWordVals = sizeof(TO) == 4 ? 1 : 2;

// Rank src's words of buffer `buf` (as mapped here) for calls of parity `parity`, (capacity, hidden)
// values in row-major order.
template <typename TO>
__device__ __forceinline__ uint64_t* comm_words(const OpArgs& a, int buf, uint32_t parity, int src) {
  return reinterpret_cast<uint64_t*>(a.bufs[buf] + a.data_off) +
         (static_cast<int64_t>(parity) * a.world + src) * a.capacity * a.hidden / kWordVals<TO>;
}

// Two words with one 16-byte access; each 64-bit element is written and read whole.
__device__ __forceinline__ void st_words2(uint64_t* p, uint64_t x, uint64_t y) {
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(x), "l"(y) : "memory");
}
__device__ __forceinline__ void ld_words2(const uint64_t* p, uint64_t& x, uint64_t& y) {
  asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(x), "=l"(y) : "l"(p) : "memory");
}

// Eight consecutive values of a partial as exchange words.
template <typename TO>
__device__ __forceinline__ void push8(uint64_t* w, float4 lo, float4 hi, uint32_t epoch) {
  const uint64_t e = static_cast<uint64_t>(epoch) << 32;
  if constexpr (sizeof(TO) == 4) {
    st_words2(w, e | __float_as_uint(lo.x), e | __float_as_uint(lo.y));
    st_words2(w + 2, e | __float_as_uint(lo.z), e | __float_as_uint(lo.w));
    st_words2(w + 4, e | __float_as_uint(hi.x), e | __float_as_uint(hi.y));
    st_words2(w + 6, e | __float_as_uint(hi.z), e | __float_as_uint(hi.w));
  } else {
    st_words2(w, e | pack2<TO>(lo.x, lo.y), e | pack2<TO>(lo.z, lo.w));
    st_words2(w + 2, e | pack2<TO>(hi.x, hi.y), e | pack2<TO>(hi.z, hi.w));
  }
}

// Four consecutive values from exchange words once they all carry `epoch`. Gives up (false) once the
// thread's deadline has passed; the deadline is set on the thread's first wait.
template <typename TO>
__device__ __forceinline__ bool pull4(const uint64_t* w, uint32_t epoch, uint64_t& deadline, float4& v) {
  uint32_t pause = 32;  // ns between polls, doubling up to 512: every finishing thread polls its own words
  while (true) {
    uint64_t x0, x1, x2 = 0, x3 = 0;
    ld_words2(w, x0, x1);
    bool ready = static_cast<uint32_t>(x0 >> 32) == epoch && static_cast<uint32_t>(x1 >> 32) == epoch;
    if constexpr (sizeof(TO) == 4) {
      ld_words2(w + 2, x2, x3);
      ready = ready && static_cast<uint32_t>(x2 >> 32) == epoch && static_cast<uint32_t>(x3 >> 32) == epoch;
    }
    if (ready) {
      if constexpr (sizeof(TO) == 4) {
        v = make_float4(__uint_as_float(static_cast<uint32_t>(x0)), __uint_as_float(static_cast<uint32_t>(x1)),
                        __uint_as_float(static_cast<uint32_t>(x2)), __uint_as_float(static_cast<uint32_t>(x3)));
      } else {
        const float2 a = unpack2<TO>(static_cast<uint32_t>(x0)), b = unpack2<TO>(static_cast<uint32_t>(x1));
        v = make_float4(a.x, a.y, b.x, b.y);
      }
      return true;
    }
    const uint64_t now = global_timer_ns();
    if (deadline == 0) deadline = now + kOpWaitNs;
    if (now > deadline) return false;
    __nanosleep(pause);
    if (pause < 512) pause <<= 1;
  }
}

// Counter increment that releases what this CTA did before its barrier and acquires what the CTAs that
// incremented before it did (device scope).
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}

__device__ __forceinline__ void red_add_f4(float* p, float4 v) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

template <typename TO>
__device__ __forceinline__ void store4(TO* p, float4 v) {
  if constexpr (std::is_same<TO, float>::value) {
    *reinterpret_cast<float4*>(p) = v;
  } else {
    *reinterpret_cast<uint2*>(p) = make_uint2(pack2<TO>(v.x, v.y), pack2<TO>(v.z, v.w));
  }
}

// Grid (hidden / 128, split, ceil(tokens / TN)), clusters (1, split, 1): cluster rank == blockIdx.y.
template <typename TO, int XP, int TN>
__global__ void __launch_bounds__(kOpThreads, 1)
    oproj_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                 const __grid_constant__ CUtensorMap xmap_lo, const OpArgs a) {
  using Cfg = OpCfg<XP, TN>;
  constexpr int NST = Cfg::kStages;
  constexpr uint32_t kIdesc = umma_idesc_f16(false, false, kOpRows, TN);
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024 - (raw_addr & 1023)) & 1023);  // stage s: weight tile, then the x planes
  float* ptile = reinterpret_cast<float*>(smem);                     // after the k loop
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NST * Cfg::kStageBytes);
  uint64_t* full = bars;             // [NST] TMA landed
  uint64_t* empty = bars + NST;      // [NST] the block's MMAs done (stage reusable)
  uint64_t* a_full = bars + 2 * NST;         // [4] weight block widened into A buffer
  uint64_t* a_free = a_full + kOpABufs;      // [4] MMAs that read A buffer done
  uint64_t* d_full = a_free + kOpABufs;      // [2] block accumulator ready
  uint64_t* d_free = d_full + 2;             // [2] block accumulator read back
  uint64_t* idle = d_free + 2;               // every MMA issued so far done (before TMEM is freed)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + Cfg::kBars);
  float* s_scale = reinterpret_cast<float*>(tmem_slot + 4);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, ks = blockIdx.y, mc = blockIdx.z;
  const int kb0 = ks * a.blocks, nkb = a.blocks;
  // the weight is read once per call unless several token tiles share it
  const uint64_t policy_w = gridDim.z > 1 ? policy_evict_last() : policy_evict_first();

  auto load_block = [&](int stage, int kb) {  // one thread
    uint8_t* st = smem + stage * Cfg::kStageBytes;
    mbar_arrive_expect_tx(&full[stage], Cfg::kStageBytes);
    tma_load_2d(st, &wmap, &full[stage], kb * 128, n_tile * kOpRows, policy_w);
  };
  auto load_x = [&](int stage, int kb) {  // one thread, after load_block of the same stage
    uint8_t* xs = smem + stage * Cfg::kStageBytes + kOpWBytes;
    const uint64_t policy_x = policy_evict_last();
    tma_load_2d(xs, &xmap, &full[stage], kb * 128, mc * TN, policy_x);
    tma_load_2d(xs + Cfg::kXBytes / 2, &xmap, &full[stage], kb * 128 + 64, mc * TN, policy_x);
    if constexpr (XP == 2) {
      tma_load_2d(xs + Cfg::kXBytes, &xmap_lo, &full[stage], kb * 128, mc * TN, policy_x);
      tma_load_2d(xs + Cfg::kXBytes + Cfg::kXBytes / 2, &xmap_lo, &full[stage], kb * 128 + 64, mc * TN, policy_x);
    }
  };

  // The producer warp owns the barriers and starts the weight loads before the CTA barrier, the issuing
  // warp allocates TMEM, the reader warps fetch the block scales meanwhile.
  const int npro = nkb < NST ? nkb : NST;
  if (warp == kOpProdWarp) {
    if (lane == 0) {
      prefetch_tensormap(&wmap);
      prefetch_tensormap(&xmap);
      if constexpr (XP == 2) prefetch_tensormap(&xmap_lo);
#pragma unroll
      for (int s = 0; s < NST; ++s) {
        mbar_init(&full[s], 1);
        mbar_init(&empty[s], 1);
      }
#pragma unroll
      for (int j = 0; j < kOpABufs; ++j) {
        mbar_init(&a_full[j], 32 * Cfg::kConvWarps);
        mbar_init(&a_free[j], 1);
      }
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        mbar_init(&d_full[j], 1);
        mbar_init(&d_free[j], 32 * Cfg::kReadWarps);
      }
      mbar_init(idle, 1);
      fence_mbar_init();
      for (int i = 0; i < npro; ++i) load_block(i, kb0 + i);  // the weight does not depend on the gating kernel
    }
    __syncwarp();
  } else if (warp == kOpIssueWarp) {
    tmem_alloc(tmem_slot, Cfg::kTmemCols);
  } else if (warp >= Cfg::kConvWarps) {
    for (int i = threadIdx.x - 32 * Cfg::kConvWarps; i < nkb; i += 32 * Cfg::kReadWarps) {
      s_scale[i] = __bfloat162float(a.scale[n_tile * a.s_sn + static_cast<int64_t>(kb0 + i) * a.s_sk]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  const uint32_t tmem = *tmem_slot;
  const uint32_t t_a = tmem, t_d = tmem + kOpABufs * 64;
  const uint32_t lane_addr = static_cast<uint32_t>(32 * (warp & 3)) << 16;  // this warp's TMEM lanes
  const int cgrp = (warp - Cfg::kConvWarps) >> 2;                         // a reader's token column group
  bool failed = false;

  float acc[Cfg::kReadCols];
#pragma unroll
  for (int t = 0; t < Cfg::kReadCols; ++t) acc[t] = 0.f;

  if (warp == kOpProdWarp) {
    // ---- TMA producer (one thread): the x tiles of the first stages, then every refill as its stage's
    // MMAs complete; at the end it waits for its last copies (a failed consumer leaves none in flight)
    if (lane == 0) {
      pdl_wait();  // x is written by the gating kernel
      for (int i = 0; i < npro; ++i) load_x(i, kb0 + i);
      int issued = npro;
      for (int b = npro; b < nkb; ++b) {
        const int s = b % NST;
        if (!mbar_wait_bounded(&empty[s], ((b / NST) - 1) & 1, kOpWaitNs)) {
          raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
          break;
        }
        load_block(s, kb0 + b);
        load_x(s, kb0 + b);
        issued = b + 1;
      }
      for (int b = issued - NST > 0 ? issued - NST : 0; b < issued; ++b) {
        if (!mbar_wait_bounded(&full[b % NST], (b / NST) & 1, kOpWaitNs)) {
          raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
          break;
        }
      }
    }
    __syncwarp();
  } else if (warp == kOpIssueWarp) {
    // ---- MMA issuer (one thread)
    if (lane == 0) {
      for (int b = 0; b < nkb && !failed; ++b) {
        const int s = b % NST, ab = b % kOpABufs, db = b & 1;
        const bool ok = mbar_wait_bounded(&full[s], (b / NST) & 1, kOpWaitNs) &&
                        mbar_wait_bounded(&a_full[ab], (b / kOpABufs) & 1, kOpWaitNs) &&
                        (b < 2 || mbar_wait_bounded(&d_free[db], ((b - 2) >> 1) & 1, kOpWaitNs));
        if (!ok) {
          failed = true;
          raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
          break;
        }
        tc_fence_after();
        const uint32_t xa = smem_u32(smem + s * Cfg::kStageBytes + kOpWBytes);
        const uint32_t d = t_d + db * Cfg::kDCols;
#pragma unroll
        for (int j = 0; j < 8; ++j) {  // k steps of 16: A columns 8j.., x half j / 4 at byte 32 (j % 4)
          const uint32_t xj = xa + (j >> 2) * (Cfg::kXBytes / 2) + (j & 3) * 32;
#pragma unroll
          for (int pl = 0; pl < XP; ++pl) {
            tc_mma_ts(d + pl * TN, t_a + ab * 64 + j * 8, umma_desc_sw128(xj + pl * Cfg::kXBytes, 16, 1024), kIdesc,
                      j > 0);
          }
        }
        tc_commit(&d_full[db]);
        tc_commit(&a_free[ab]);
        tc_commit(&empty[s]);
      }
      tc_commit(idle);
    }
    __syncwarp();
  } else if (warp < Cfg::kConvWarps) {
    // ---- converter warps: row 32 (warp % 4) + lane, 16-byte units [part * kConvUnits, +kConvUnits) of it
    const int r = 32 * (warp & 3) + lane, part = warp >> 2;
    for (int b = 0; b < nkb; ++b) {
      const int s = b % NST, ab = b % kOpABufs;
      bool ok = !failed && mbar_wait_bounded(&full[s], (b / NST) & 1, kOpWaitNs) &&
                (b < kOpABufs || mbar_wait_bounded(&a_free[ab], ((b - kOpABufs) / kOpABufs) & 1, kOpWaitNs));
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && !failed) {
        if (lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
        failed = true;
      }
      if (!failed) {
        tc_fence_after();
        // weight row r: 16-byte units u of the 128-byte swizzled row sit at (u ^ (r % 8)) * 16
        const uint32_t row = smem_u32(smem + s * Cfg::kStageBytes) + r * 128;
#pragma unroll
        for (int h = 0; h < Cfg::kConvUnits / 2; ++h) {  // 32 bytes (32 k) -> 16 columns per step
          uint32_t w[16];
#pragma unroll
          for (int u2 = 0; u2 < 2; ++u2) {
            const int u = part * Cfg::kConvUnits + 2 * h + u2;
            const uint4 v = lds128(row + ((static_cast<uint32_t>(u) ^ (r & 7)) << 4));
            e4m3x4_to_f16x2(v.x, w[8 * u2 + 0], w[8 * u2 + 1]);
            e4m3x4_to_f16x2(v.y, w[8 * u2 + 2], w[8 * u2 + 3]);
            e4m3x4_to_f16x2(v.z, w[8 * u2 + 4], w[8 * u2 + 5]);
            e4m3x4_to_f16x2(v.w, w[8 * u2 + 6], w[8 * u2 + 7]);
          }
          tmem_st16(t_a + lane_addr + ab * 64 + (part * Cfg::kConvUnits + 2 * h) * 8, w);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(&a_full[ab]);
    }
  } else {
    // ---- reader warps: row 32 (warp % 4) + lane, token columns [cgrp * kReadCols, +kReadCols) of every
    // block accumulator, times the block's scale
    for (int c = 0; c < nkb; ++c) {
      const int db = c & 1;
      bool ok = !failed && mbar_wait_bounded(&d_full[db], (c >> 1) & 1, kOpWaitNs);
      ok = __all_sync(0xffffffffu, ok);
      if (ok) {
        tc_fence_after();
        const float sc = s_scale[c];
#pragma unroll
        for (int q = 0; q < Cfg::kReadCols / 32; ++q) {
#pragma unroll
          for (int pl = 0; pl < XP; ++pl) {  // the hi plane, then the lo plane (stored times 2^11)
            uint32_t v[32];
            tmem_ld32(t_d + lane_addr + db * Cfg::kDCols + pl * TN + cgrp * Cfg::kReadCols + q * 32, v);
            tmem_ld_wait();
            const float f = pl == 0 ? sc : sc * (1.f / kLoScale);
#pragma unroll
            for (int t = 0; t < 32; ++t) acc[q * 32 + t] = fmaf(f, __uint_as_float(v[t]), acc[q * 32 + t]);
          }
        }
      } else if (!failed) {
        if (lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
        failed = true;
      }
      tc_fence_before();
      mbar_arrive(&d_free[db]);
    }
  }

  // ---- this CTA's partial tile [token][hidden row] (over the drained stages), added into the tile's fp32
  // sum; the tile's last CTA rounds the sum and stores or pushes it
  __syncthreads();  // every MMA has completed (the readers saw the last block's accumulator)
  if (warp == kOpIssueWarp) {
    if (lane == 0 && !mbar_wait_bounded(idle, 0, kOpWaitNs)) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  } else if (warp >= Cfg::kConvWarps && warp < kOpIssueWarp) {
    const int r = 32 * (warp & 3) + lane;
#pragma unroll
    for (int t = 0; t < Cfg::kReadCols; ++t) ptile[(cgrp * Cfg::kReadCols + t) * kOpPitch + r] = acc[t];
  }
  __syncthreads();
  pdl_wait();  // the sums were cleared by the gating kernel
  const int64_t tile = static_cast<int64_t>(mc) * gridDim.x + n_tile;
  float* tsum = a.sums + static_cast<int64_t>(mc) * TN * a.hidden + static_cast<int64_t>(n_tile) * kOpRows;
  const int valid = a.tokens - mc * TN < TN ? a.tokens - mc * TN : TN;
  const bool alone = a.split == 1;  // the tile has one CTA: its partial is the sum
  if (!alone) {
    for (int it = threadIdx.x; it < valid * (kOpRows / 4); it += kOpThreads) {
      const int tok = it / (kOpRows / 4), nl = 4 * (it - tok * (kOpRows / 4));
      red_add_f4(tsum + static_cast<int64_t>(tok) * a.hidden + nl,
                 *reinterpret_cast<const float4*>(ptile + tok * kOpPitch + nl));
    }
    // every thread's reductions precede thread 0's acquire-release increment through the barrier (release
    // is cumulative), and the tile's last CTA reads the sums after its own increment acquired all of them
    __syncthreads();
    __shared__ int s_last;
    if (threadIdx.x == 0) s_last = atom_add_acq_rel_gpu(&a.counters[tile], 1u) == static_cast<uint32_t>(a.split - 1);
    __syncthreads();
    if (!s_last) return;
  }
  const uint32_t epoch = a.world > 1 ? comm_state(a)[0] + 1u : 0u;
  auto tile_sum = [&](int tok, int nl) {
    return alone ? *reinterpret_cast<const float4*>(ptile + tok * kOpPitch + nl)
                 : __ldcg(reinterpret_cast<const float4*>(tsum + static_cast<int64_t>(tok) * a.hidden + nl));
  };
  if (a.world == 1) {
    TO* out = static_cast<TO*>(a.out);
    for (int it = threadIdx.x; it < valid * (kOpRows / 4); it += kOpThreads) {
      const int tok = it / (kOpRows / 4), nl = 4 * (it - tok * (kOpRows / 4));
      const int64_t token = static_cast<int64_t>(mc) * TN + tok;
      store4(out + token * a.o_st + static_cast<int64_t>(n_tile) * kOpRows + nl, tile_sum(tok, nl));
    }
  } else {
    // eight values = 32 or 64 bytes of words per store group (rows are hidden values long, a multiple of 128)
    for (int it = threadIdx.x; it < valid * (kOpRows / 8); it += kOpThreads) {
      const int tok = it / (kOpRows / 8), nl = 8 * (it - tok * (kOpRows / 8));
      const int64_t off = (static_cast<int64_t>(mc) * TN + tok) * a.hidden + static_cast<int64_t>(n_tile) * kOpRows + nl;
      const float4 lo = tile_sum(tok, nl), hi = tile_sum(tok, nl + 4);
      for (int p = 0; p < a.world; ++p) push8<TO>(comm_words<TO>(a, p, epoch & 1u, a.rank) + off / kWordVals<TO>, lo, hi, epoch);
    }
  }
}

// Grid (hidden / 128, kFinishSlices, token tiles): CTA (x, y, z) finishes row quads
// [y * 32 / kFinishSlices, (y + 1) * 32 / kFinishSlices) of the tile that oproj_kernel's last CTA of tile
// (x, z) pushed.
template <typename TO>
__global__ void __launch_bounds__(256) oproj_finish_kernel(const OpArgs a) {
  pdl_wait();  // this rank's own partial comes from oproj_kernel
  const int n_tile = blockIdx.x, mc = blockIdx.z;
  constexpr int kQuads = kOpRows / 4;
  const int q0 = blockIdx.y * kQuads / gridDim.y, nq = (blockIdx.y + 1) * kQuads / gridDim.y - q0;
  uint32_t* state = comm_state(a);
  const uint32_t epoch = state[0] + 1u;
  uint64_t deadline = 0;
  uint32_t missing = 0;  // peers whose words never carried the epoch (bit per rank)
  TO* out = static_cast<TO*>(a.out);
  for (int it = threadIdx.x; it < a.tn * nq; it += blockDim.x) {
    const int tok = it / nq;
    const int64_t token = static_cast<int64_t>(mc) * a.tn + tok;
    if (token >= a.tokens) continue;
    const int64_t n = static_cast<int64_t>(n_tile) * kOpRows + 4 * (q0 + it - tok * nq);
    const int64_t off = token * a.hidden + n;
    float4 sum = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int p = 0; p < a.world; ++p) {  // rank order
      if (missing & (1u << p)) continue;  // a peer that never arrived: its words are stale (the error word says so)
      float4 v;
      if (!pull4<TO>(comm_words<TO>(a, a.rank, epoch & 1u, p) + off / kWordVals<TO>, epoch, deadline, v)) {
        missing |= 1u << p;
        continue;
      }
      sum.x += v.x; sum.y += v.y; sum.z += v.z; sum.w += v.w;
    }
    store4(out + token * a.o_st + n, sum);
  }
  if (missing) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
  // the last CTA to finish publishes this call's epoch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const uint32_t total = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(&state[1], 1u) == total - 1u) {
      state[1] = 0u;
      __threadfence();
      state[0] = epoch;
    }
  }
}

// ---- host ------------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 map_encoder() {
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

// 2-D map of a row-major (rows, cols) matrix with `row_bytes` between rows, box (box_cols, box_rows),
// 128-byte swizzle (box_cols * element size == 128).
int encode_matrix_map(CUtensorMap* map, CUtensorMapDataType type, const void* base, int64_t cols, int64_t rows,
                      int64_t row_bytes, uint32_t box_cols, uint32_t box_rows) {
  auto fn = map_encoder();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return PKV_ERR_CUDA;
  }
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}


// The projection's part of the workspace after the two f16 planes: fp32 split-k sums for (tokens, hidden)
// (only valid tokens are ever added or read), then one counter per tile of 32 tokens.
int64_t sums_bytes(int64_t tokens, int64_t hidden) { return align_up(std::max<int64_t>(tokens, 1) * hidden * 4, 256); }
int64_t counters_bytes(int64_t tokens, int64_t hidden) {
  return align_up((hidden / kOpRows) * ceil_div(std::max<int64_t>(tokens, 1), kOpMinTokens) * 4, 256);
}

int64_t comm_data_offset() { return align_up(kCommHeader, 256); }

template <typename TH, typename TG>
int launch_gate(const GateArgs& g, bool chained, cudaStream_t s) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(ceil_div(g.k / 8, 256)),
                     static_cast<unsigned>(std::min<int64_t>(g.tokens, 65535)));
  cfg.blockDim = dim3(256);
  cfg.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = chained ? 1 : 0;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  const cudaError_t e = std::is_same<typename Promote<TH, TG>::type, float>::value
                            ? cudaLaunchKernelEx(&cfg, oproj_gate_kernel<TH, TG, 2>, g)
                            : cudaLaunchKernelEx(&cfg, oproj_gate_kernel<TH, TG, 1>, g);
  return cuda_status(e, "oproj_gate_kernel launch");
}

template <typename TH>
int dispatch_gate(int gate_dtype, const GateArgs& g, bool chained, cudaStream_t s) {
  switch (gate_dtype) {
    case PKV_DTYPE_F32: return launch_gate<TH, float>(g, chained, s);
    case PKV_DTYPE_F16: return launch_gate<TH, __half>(g, chained, s);
    default: return launch_gate<TH, __nv_bfloat16>(g, chained, s);
  }
}

template <typename TO, int XP, int TN>
cudaError_t set_smem_attr() {
  return prepare_kernel(reinterpret_cast<const void*>(oproj_kernel<TO, XP, TN>), OpCfg<XP, TN>::kSmem);
}

template <typename TO, int XP, int TN>
int launch_oproj(const OpArgs& a, const CUtensorMap& wmap, const CUtensorMap& xmap, const CUtensorMap& xmap_lo,
                 dim3 grid, bool main_phase, bool finish_phase, cudaStream_t s) {
  const cudaError_t attr_err = set_smem_attr<TO, XP, TN>();
  if (attr_err != cudaSuccess) return cuda_status(attr_err, "oproj_kernel shared memory attribute");
  if (main_phase) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kOpThreads);
    cfg.dynamicSmemBytes = OpCfg<XP, TN>::kSmem;
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, oproj_kernel<TO, XP, TN>, wmap, xmap, xmap_lo, a);
    if (e != cudaSuccess) return cuda_status(e, "oproj_kernel launch");
  }
  if (finish_phase && a.world > 1) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(grid.x, kFinishSlices, grid.z);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr.val.programmaticStreamSerializationAllowed = main_phase ? 1 : 0;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, oproj_finish_kernel<TO>, a);
    if (e != cudaSuccess) return cuda_status(e, "oproj_finish_kernel launch");
  }
  return PKV_OK;
}

template <typename TO>
int dispatch_planes(bool two_planes, int tn, const OpArgs& a, const CUtensorMap& wmap, const CUtensorMap& xmap,
                    const CUtensorMap& xmap_lo, dim3 grid, bool main_phase, bool finish_phase, cudaStream_t s) {
  if (two_planes) {
    return tn == 64 ? launch_oproj<TO, 2, 64>(a, wmap, xmap, xmap_lo, grid, main_phase, finish_phase, s)
                    : launch_oproj<TO, 2, 32>(a, wmap, xmap, xmap_lo, grid, main_phase, finish_phase, s);
  }
  if (tn == 128) return launch_oproj<TO, 1, 128>(a, wmap, xmap, xmap_lo, grid, main_phase, finish_phase, s);
  return tn == 64 ? launch_oproj<TO, 1, 64>(a, wmap, xmap, xmap_lo, grid, main_phase, finish_phase, s)
                  : launch_oproj<TO, 1, 32>(a, wmap, xmap, xmap_lo, grid, main_phase, finish_phase, s);
}

bool aligned(const void* p, int64_t bytes) { return (reinterpret_cast<uintptr_t>(p) % bytes) == 0; }

int device_sm_count() {
  int dev = 0, sms = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int64_t pkv_o_proj_workspace_size(int64_t num_tokens, int64_t k_local, int64_t hidden) {
  if (num_tokens < 0 || k_local < 0 || hidden < 0) return -1;
  // hi and lo planes of f16 activations, fp32 split-k sums, tile counters
  return 2 * align_up(num_tokens * k_local * 2, 256) + sums_bytes(num_tokens, hidden) +
         counters_bytes(num_tokens, hidden);
}

extern "C" int64_t pkv_o_proj_comm_bytes(int world, int64_t capacity_tokens, int64_t hidden, int out_dtype) {
  if (world < 1 || world > kOpMaxWorld || capacity_tokens < 1 || hidden < kOpRows || hidden % kOpRows != 0 ||
      dtype_size(out_dtype) == 0) {
    return -1;
  }
  // two call parities x world ranks x (capacity, hidden) values, as 8-byte words of two 16-bit values (or one
  // fp32 value) and the epoch: twice the values' own bytes
  return comm_data_offset() + 2ll * world * capacity_tokens * hidden * 2 * dtype_size(out_dtype);
}

extern "C" int pkv_gated_o_proj(const void* heads, int64_t h_stride_batch, int64_t h_stride_head, int64_t h_stride_seq,
                                int heads_dtype, const void* gate, int64_t g_stride_batch, int64_t g_stride_seq,
                                int gate_dtype, int64_t batch, int64_t seq_len, int64_t num_heads, int64_t head_dim,
                                const void* weight, int64_t w_stride_row, const void* scale_inv, int64_t s_stride_row,
                                int64_t s_stride_col, int64_t hidden, void* out, int64_t o_stride_token, int out_dtype,
                                void* workspace, int64_t workspace_bytes, int rank, int world,
                                void* const* comm_buffers, int64_t comm_capacity_tokens, int phases,
                                int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE(batch >= 0 && seq_len >= 1 && num_heads >= 1 && head_dim >= 1, "bad shape");
  PKV_REQUIRE(dtype_size(heads_dtype) && dtype_size(gate_dtype) && dtype_size(out_dtype), "unsupported dtype");
  PKV_REQUIRE(world >= 1 && world <= kOpMaxWorld && rank >= 0 && rank < world, "rank must be in [0, world), world <= 8");
  const bool chained = (phases & PKV_OPROJ_CHAINED) != 0;
  phases &= ~PKV_OPROJ_CHAINED;
  PKV_REQUIRE(phases >= 1 && phases <= 3,
              "phases must be 1 (compute + push), 2 (finish) or 3 (both), optionally | PKV_OPROJ_CHAINED");
  const int64_t k = num_heads * head_dim, tokens = batch * seq_len;
  PKV_UNSUPPORTED(k % 128 == 0, "num_heads * head_dim must be a multiple of 128 (the weight's scale blocks)");
  PKV_UNSUPPORTED(hidden >= kOpRows && hidden % kOpRows == 0, "hidden must be a positive multiple of 128");
  PKV_UNSUPPORTED(head_dim % 8 == 0, "head_dim must be a multiple of 8");
  PKV_REQUIRE(k < (1ll << 31) && hidden < (1ll << 31) && tokens < (1ll << 31), "sizes must fit in 32 bits");
  if (tokens == 0) return PKV_OK;
  PKV_REQUIRE(heads && gate && weight && scale_inv && out, "null pointer");
  PKV_REQUIRE(aligned(heads, 16) && aligned(gate, 16) && h_stride_batch % 8 == 0 && h_stride_head % 8 == 0 &&
                  h_stride_seq % 8 == 0 && g_stride_batch % 8 == 0 && g_stride_seq % 8 == 0,
              "heads and gate need 16-byte aligned rows (strides multiples of 8 elements)");
  PKV_REQUIRE(aligned(weight, 16) && w_stride_row % 16 == 0 && w_stride_row >= k, "weight rows must be 16-byte aligned");
  PKV_REQUIRE(aligned(out, 16) && o_stride_token % 4 == 0 && o_stride_token >= hidden,
              "out rows must be 16-byte aligned (token stride a multiple of 4)");
  PKV_REQUIRE(workspace != nullptr && aligned(workspace, 256) &&
                  workspace_bytes >= pkv_o_proj_workspace_size(tokens, k, hidden),
              "workspace too small or not 256-byte aligned");
  if (world > 1) {
    PKV_REQUIRE(comm_buffers != nullptr, "comm_buffers required when world > 1");
    for (int p = 0; p < world; ++p) PKV_REQUIRE(comm_buffers[p] != nullptr && aligned(comm_buffers[p], 256), "bad comm buffer");
    PKV_REQUIRE(tokens <= comm_capacity_tokens, "more tokens than the exchange buffers hold");
  }
  auto s = static_cast<cudaStream_t>(stream);
  const bool main_phase = phases & 1, finish_phase = phases & 2;
  bump_stat(kStatGatedOProj);
  // fp32 products (torch promotes mixed types to fp32) travel as two f16 planes
  const bool two_planes = heads_dtype == PKV_DTYPE_F32 || gate_dtype == PKV_DTYPE_F32 || heads_dtype != gate_dtype;
  const int64_t plane_bytes = align_up(tokens * k * 2, 256);

  // launch shape of the projection (the gating kernel clears the split-k sums only when split > 1)
  OpArgs a{};
  a.scale = static_cast<const __nv_bfloat16*>(scale_inv);
  a.s_sn = s_stride_row; a.s_sk = s_stride_col;
  a.tokens = static_cast<int32_t>(tokens);
  a.hidden = static_cast<int32_t>(hidden);
  a.k = static_cast<int32_t>(k);
  // token tile (the MMA's N): 32 for at most 32 tokens, 64 up to 64 tokens (or with two planes), else 128;
  // split-k factor: the largest divisor of the 128-k block count (<= 8) that keeps the CTAs within one wave
  // of the SMs (one CTA fits an SM)
  const int kblocks = static_cast<int>(k / 128);
  const int tn = tokens <= 32 ? 32 : (tokens <= 64 || two_planes) ? 64 : 128;
  const int64_t tiles = (hidden / kOpRows) * ceil_div(tokens, tn);
  int split = 1;
  for (int c = kOpMaxSplit; c >= 1; --c) {
    if (kblocks % c == 0 && tiles * c <= device_sm_count()) {
      split = c;
      break;
    }
  }
  constexpr int kMaxBlocks = OpCfg<1, 64>::kMaxBlocks;
  PKV_UNSUPPORTED(kblocks / split <= kMaxBlocks, "num_heads * head_dim too large for one call");
  a.split = split;
  a.blocks = kblocks / split;
  a.tn = tn;
  a.sums = reinterpret_cast<float*>(static_cast<char*>(workspace) + 2 * plane_bytes);
  a.counters = reinterpret_cast<uint32_t*>(static_cast<char*>(workspace) + 2 * plane_bytes + sums_bytes(tokens, hidden));

  // 1. gating
  if (main_phase) {
    GateArgs g{};
    g.heads = heads;
    g.h_sb = h_stride_batch; g.h_sh = h_stride_head; g.h_ss = h_stride_seq;
    g.gate = gate;
    g.g_sb = g_stride_batch; g.g_ss = g_stride_seq;
    g.seq_len = static_cast<int32_t>(seq_len);
    g.head_dim = static_cast<int32_t>(head_dim);
    g.k = static_cast<int32_t>(k);
    g.hd_shift = (head_dim & (head_dim - 1)) == 0 ? __builtin_ctzll(static_cast<uint64_t>(head_dim)) : -1;
    g.tokens = tokens;
    g.x = static_cast<__half*>(workspace);
    g.plane = plane_bytes / 2;
    g.clear = reinterpret_cast<float4*>(static_cast<char*>(workspace) + 2 * plane_bytes);
    g.clear_vec4 = split > 1 ? (sums_bytes(tokens, hidden) + counters_bytes(tokens, hidden)) / 16 : 0;
    int st;
    switch (heads_dtype) {
      case PKV_DTYPE_F32: st = dispatch_gate<float>(gate_dtype, g, chained, s); break;
      case PKV_DTYPE_F16: st = dispatch_gate<__half>(gate_dtype, g, chained, s); break;
      default: st = dispatch_gate<__nv_bfloat16>(gate_dtype, g, chained, s); break;
    }
    if (st != PKV_OK) return st;
  }

  a.out = out;
  a.o_st = o_stride_token;
  a.world = world;
  a.rank = rank;
  for (int p = 0; p < world; ++p) a.bufs[p] = world > 1 ? static_cast<char*>(comm_buffers[p]) : nullptr;
  a.capacity = comm_capacity_tokens;
  a.data_off = comm_data_offset();
  a.error_flag = error_flag;
  const dim3 grid(static_cast<unsigned>(hidden / kOpRows), static_cast<unsigned>(split),
                  static_cast<unsigned>(ceil_div(tokens, tn)));
  CUtensorMap wmap{}, xmap{}, xmap_lo{};
  if (main_phase) {
    int st = encode_matrix_map(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, weight, k, hidden, w_stride_row, 128, kOpRows);
    if (st != PKV_OK) return st;
    st = encode_matrix_map(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, workspace, k, tokens, k * 2, 64, tn);
    if (st != PKV_OK) return st;
    xmap_lo = xmap;
    if (two_planes) {
      st = encode_matrix_map(&xmap_lo, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, static_cast<char*>(workspace) + plane_bytes, k,
                             tokens, k * 2, 64, tn);
      if (st != PKV_OK) return st;
    }
  }
  switch (out_dtype) {
    case PKV_DTYPE_F32: return dispatch_planes<float>(two_planes, tn, a, wmap, xmap, xmap_lo, grid, main_phase, finish_phase, s);
    case PKV_DTYPE_F16: return dispatch_planes<__half>(two_planes, tn, a, wmap, xmap, xmap_lo, grid, main_phase, finish_phase, s);
    default: return dispatch_planes<__nv_bfloat16>(two_planes, tn, a, wmap, xmap, xmap_lo, grid, main_phase, finish_phase, s);
  }
}

// ---- exchange buffers shared between processes (CUDA IPC) ------------------------------------------------------
extern "C" int64_t pkv_ipc_handle_bytes() { return static_cast<int64_t>(sizeof(cudaIpcMemHandle_t)); }

extern "C" int pkv_ipc_alloc(int64_t bytes, void** ptr, void* handle) {
  clear_error();
  PKV_REQUIRE(bytes > 0 && ptr != nullptr, "bad arguments");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, static_cast<size_t>(bytes));
  if (e != cudaSuccess) return cuda_status(e, "cudaMalloc of the exchange buffer");
  e = cudaMemset(p, 0, static_cast<size_t>(bytes));
  if (e == cudaSuccess && handle != nullptr) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_status(e, "exchange buffer setup");
  }
  *ptr = p;
  return PKV_OK;
}

extern "C" int pkv_ipc_open(const void* handle, void** ptr) {
  clear_error();
  PKV_REQUIRE(handle != nullptr && ptr != nullptr, "bad arguments");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
}

extern "C" int pkv_ipc_close(void* ptr) {
  clear_error();
  return cuda_status(cudaIpcCloseMemHandle(ptr), "cudaIpcCloseMemHandle");
}

extern "C" int pkv_ipc_free(void* ptr) {
  clear_error();
  return cuda_status(cudaFree(ptr), "cudaFree of the exchange buffer");
}
