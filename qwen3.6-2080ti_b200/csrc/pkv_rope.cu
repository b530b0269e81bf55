// Fused q/k RMSNorm + partial rotary embedding + K/V append (the per-layer step in front of paged
// attention).
//
// The reference runs, per full-attention layer (src/tp_runtime.py:510-525, batched decode :2461-2483):
//   query = rms_norm(query, q_norm); key = rms_norm(key, k_norm)            (src/reference_ops.py:166-169)
//   cos, sin = rotary_embeddings(positions)                                 (src/reference_ops.py:203-212)
//   query, key = apply_rotary_pos_emb(query, key, cos, sin)                 (src/reference_ops.py:215-224)
//   key, value = _repeat_kv(...)[TP slice]; cache.append_blocks(key, value) (src/decode_state.py:271-293)
// as separate torch launches with the new K/V round-tripping through memory. Here one launch does it
// all. A token has Hq query rows (written to q_out), Hkv key rows and Hkv value rows (the post-RoPE key
// and the raw value written straight into the token's slot; no repeated heads). A warp processes a row
// with each lane holding D/32 consecutive elements in registers from load to store: the rotary partner
// of a lane's run (rotary_dim / 2 elements away) is another lane's whole run and comes by shuffle.
//
// Arithmetic follows the reference's dtype semantics:
//   rms_norm   fp32 mean of squares, x * (1 / sqrt(mean + eps)) * (1 + w) in fp32, rounded to dtype
//   rotary     on the first rotary_dim elements: out = rnd(rnd(x * cos) + rnd(rotate_half(x) * sin)),
//              rotate_half(x)_i = -x_{i + r/2} for i < r/2, x_{i - r/2} otherwise; cos/sin rows come
//              from the caller's table (built as rotary_embeddings builds them, already in dtype)
// where rnd rounds to the tensor dtype (torch computes each dtype op in fp32 and rounds), so given the
// same normalised values and table the rotary part is bit-identical; the mean of squares is summed in a
// different order than torch's reduction, which can move a normalised value by one unit in the last
// place.
#include <cmath>
#include <type_traits>

#include "pkv_common.cuh"

namespace pkv {
namespace {

// Packed pairs of a 16-bit dtype: each result is the exact product / sum rounded once to nearest even,
// which is what torch's dtype ops give (the exact product or sum of two 16-bit values is rounded to
// fp32 without loss of the tie decision, then rounded to the dtype).
template <typename T>
__device__ __forceinline__ uint32_t mul2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  } else {
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  }
  return r;
}
template <typename T>
__device__ __forceinline__ uint32_t add2_rn(uint32_t a, uint32_t b) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  } else {
    asm("add.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  }
  return r;
}

// A packed pair of 16-bit values -> the fp32 pair (as one 64-bit register pair), and back with one
// round-to-nearest-even conversion.
template <typename T>
__device__ __forceinline__ uint64_t widen2(uint32_t w) {
  uint64_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("{\n\t.reg .b32 lo, hi;\n\tshl.b32 lo, %1, 16;\n\tand.b32 hi, %1, 0xffff0000;\n\tmov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r) : "r"(w));
  } else {
    asm("{\n\t.reg .b16 a, b;\n\t.reg .f32 lo, hi;\n\tmov.b32 {a, b}, %1;\n\tcvt.f32.f16 lo, a;\n\tcvt.f32.f16 hi, b;\n\t"
        "mov.b64 %0, {lo, hi};\n\t}"
        : "=l"(r) : "r"(w));
  }
  return r;
}
template <typename T>
__device__ __forceinline__ uint32_t narrow2(uint64_t v) {
  uint32_t r;
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    asm("{\n\t.reg .f32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tcvt.rn.bf16x2.f32 %0, hi, lo;\n\t}" : "=r"(r) : "l"(v));
  } else {
    asm("{\n\t.reg .f32 lo, hi;\n\tmov.b64 {lo, hi}, %1;\n\tcvt.rn.f16x2.f32 %0, hi, lo;\n\t}" : "=r"(r) : "l"(v));
  }
  return r;
}

template <typename I>
struct RopeArgs {
  const void* q;
  int64_t q_st, q_sh;
  const void* k;
  int64_t k_st, k_sh;
  const void* v;
  int64_t v_st, v_sh;
  const void* q_weight;
  const void* k_weight;
  float eps;
  const void* cos_sin;  // (max_position, 2 * rotary_dim): cos then sin
  int64_t max_position;
  int32_t rotary_dim;
  const I* positions;
  int64_t position_offset;
  const int64_t* slots;
  void* key_pool;
  void* value_pool;
  int64_t num_slots;  // num_pages * block_size
  int64_t block_size, sp, sh, ss;
  int32_t bs_shift;   // log2(block_size) when it is a power of two, else -1
  void* q_out;
  int64_t qo_st, qo_sh;
  int64_t num_tokens;
  int32_t num_q_heads, num_kv_heads;
  int32_t* error_flag;
};

constexpr int kNrWarps = 4;       // warps per block
constexpr int kNrStages = 3;      // row groups per warp: one being processed, two in flight
constexpr int kNrBarBytes = 32;   // per warp: one mbarrier per stage
constexpr uint64_t kNrWaitNs = 2000000000ull;  // bounded waits: 2 s

// A row of D elements is held by LPR lanes (16 when D <= 256, so that a warp works on two rows at
// once, else 32), EPL = D / LPR elements each, as CPL chunks of CE consecutive elements (16 bytes, or
// the whole run when it is shorter): lane sl of its row holds chunks sl, sl + LPR, sl + 2 LPR, ...
template <typename T, int EPL, int LPR>
struct NrConfig {
  static constexpr int kCE = 16 / static_cast<int>(sizeof(T)) < EPL ? 16 / static_cast<int>(sizeof(T)) : EPL;
  static constexpr int kCPL = EPL / kCE;
  static constexpr int kChunkBytes = kCE * static_cast<int>(sizeof(T));
  static constexpr int kRowElems = EPL * LPR;
  static constexpr int kRowBytes = kRowElems * static_cast<int>(sizeof(T));
  static constexpr int kRows = kRowBytes >= 2048 ? 2 : 2048 / kRowBytes;  // rows per group (even)
  static constexpr int kRowsPerStep = 32 / LPR;
  static_assert(kChunkBytes % 4 == 0 && kCE % 2 == 0, "chunks of whole words");
};

// Blocks per SM the register allocation is sized for: 8 (64 registers) where a lane's run fits, fewer
// for the long fp32 and 1024-element runs.
template <typename T, int EPL>
constexpr int nr_min_blocks() {
  return EPL >= 32 ? 4 : (sizeof(T) == 4 && EPL >= 16 ? 6 : 8);
}

// Stages `cnt` rows of kRowBytes from `src` (rows `stride` elements apart) at `dst`: one bulk copy when
// the rows are adjacent, else one per row.
template <typename T, int kRowBytes>
__device__ __forceinline__ void stage_rows(uint8_t* dst, const T* src, int cnt, int64_t stride, bool adjacent,
                                           uint64_t* bar) {
  if (cnt <= 0) return;
  if (adjacent) {
    bulk_load(dst, src, static_cast<uint32_t>(cnt * kRowBytes), bar);
  } else {
    for (int r = 0; r < cnt; ++r) bulk_load(dst + r * kRowBytes, src + r * stride, kRowBytes, bar);
  }
}

// Shared-memory loads by 32-bit shared-window address (volatile: they stay after the mbarrier waits).
template <int kBytes>
__device__ __forceinline__ void lds_at(uint32_t addr, uint32_t* w) {
  if constexpr (kBytes == 16) {
    asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]) : "r"(addr));
  } else if constexpr (kBytes == 8) {
    asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(w[0]), "=r"(w[1]) : "r"(addr));
  } else {
    asm volatile("ld.shared.b32 %0, [%1];" : "=r"(w[0]) : "r"(addr));
  }
}
__device__ __forceinline__ void lds_pairs2(uint32_t addr, uint64_t& a, uint64_t& b) {
  asm volatile("ld.shared.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}
__device__ __forceinline__ uint64_t lds_pair(uint32_t addr) {
  uint64_t a;
  asm volatile("ld.shared.b64 %0, [%1];" : "=l"(a) : "r"(addr));
  return a;
}

template <int kBytes>
__device__ __forceinline__ void lds_words(const void* p, uint32_t* w) {
  if constexpr (kBytes == 16) {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (kBytes == 8) {
    const uint2 v = *reinterpret_cast<const uint2*>(p);
    w[0] = v.x; w[1] = v.y;
  } else {
    w[0] = *reinterpret_cast<const uint32_t*>(p);
  }
}
template <int kBytes>
__device__ __forceinline__ void st_words(void* p, const uint32_t* w) {
  if constexpr (kBytes == 16) {
    *reinterpret_cast<uint4*>(p) = make_uint4(w[0], w[1], w[2], w[3]);
  } else if constexpr (kBytes == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(w[0], w[1]);
  } else {
    *reinterpret_cast<uint32_t*>(p) = w[0];
  }
}
// A token has `rows` = Hq query rows, Hkv key rows, Hkv value rows, cut into groups of up to kRows rows.
// Warp w owns the contiguous range of groups [n_begin, n_end) (the token index is divided out once and
// then advanced incrementally) and stages each group in a private kNrStages-deep ring of shared
// memory, two groups ahead of the one it processes: lane 0 issues one bulk copy per adjacent run of
// query, key or value rows plus the token's cos/sin row, completed on the stage's mbarrier. Positions
// and slots are read and validated 32 tokens at a time, one token per lane. Processing reads each row
// from shared memory once: query/key rows are normalised and rotated in registers and stored, value
// rows copied, kRowsPerStep rows per warp step. Stage layout: kRows rows | cos/sin row (2 * rotary_dim
// elements) | {position, slot}.
template <typename T, typename I, int EPL, int LPR>
__global__ void __launch_bounds__(kNrWarps * 32, nr_min_blocks<T, EPL>()) norm_rope_append_kernel(const RopeArgs<I> a) {
  using Cfg = NrConfig<T, EPL, LPR>;
  constexpr int R = Cfg::kRows, CE = Cfg::kCE, CPL = Cfg::kCPL, CB = Cfg::kChunkBytes;
  constexpr int kRowBytes = Cfg::kRowBytes, D = Cfg::kRowElems, RPS = Cfg::kRowsPerStep;
  constexpr int WPC = CB / 4;  // words per chunk
  extern __shared__ __align__(16) uint8_t nr_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = lane / LPR, sl = lane % LPR;  // which row of the step, lane within the row
  const int table_bytes = 2 * a.rotary_dim * static_cast<int>(sizeof(T));
  const int stage_bytes = R * kRowBytes + table_bytes + 16;
  // (1 + w) in fp32, query norm then key norm, each in the order the lanes read it: the float4 holding
  // elements (sl + LPR j) CE + 4 u .. + 3 at float4 index (j (CE / 4) + u) LPR + sl (runs shorter than
  // four elements: float2 pairs in the same order)
  float* w1 = reinterpret_cast<float*>(nr_smem);
  uint64_t* bars = reinterpret_cast<uint64_t*>(nr_smem + 2 * D * 4 + warp * kNrBarBytes);
  uint8_t* ring = nr_smem + 2 * D * 4 + kNrWarps * kNrBarBytes + warp * (kNrStages * stage_bytes);
  constexpr int kW = CE >= 4 ? 4 : 2;  // floats per weight load
  for (int e = threadIdx.x; e < D; e += blockDim.x) {
    const int c = e / CE, i = e % CE;  // chunk c = sl + LPR j
    const int at = ((c / LPR) * (CE / kW) + i / kW) * LPR * kW + (c % LPR) * kW + i % kW;
    w1[at] = 1.f + Elem<T>::to_f(static_cast<const T*>(a.q_weight)[e]);
    w1[D + at] = 1.f + Elem<T>::to_f(static_cast<const T*>(a.k_weight)[e]);
  }
  __syncthreads();
  const int hq = a.num_q_heads, hkv = a.num_kv_heads;
  const int rows = hq + 2 * hkv;
  const int per_token = (rows + R - 1) / R;  // groups per token
  // groups, tokens, slots and positions are all below 2^31 (checked on the host)
  const int64_t groups = a.num_tokens * per_token;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kNrWarps + warp;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * kNrWarps;
  const int n_begin = static_cast<int>(groups * gw / nw), n_count = static_cast<int>(groups * (gw + 1) / nw) - n_begin;
  if (n_count <= 0) return;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < kNrStages; ++s) mbar_init(&bars[s], 1);
    fence_mbar_init();
  }
  __syncwarp();

  // rotary partners: element e < r / 2 pairs with e + r / 2. When the rotary elements all sit in the
  // lanes' first chunks and r / 2 is a whole number of chunks, a lane's partner chunk is the first chunk
  // of lane sl -+ dc of the same row (one shuffle); otherwise the rotation goes through shared memory.
  const int r = a.rotary_dim;
  const bool rot_in_regs = r > 0 && r <= LPR * CE && (r / 2) % CE == 0;
  const int rot_lanes = rot_in_regs ? r / CE : 0, dc = rot_lanes / 2;
  const int partner = half * LPR + (sl < dc ? sl + dc : (sl < rot_lanes ? sl - dc : sl));
  const bool q_adj = a.q_sh * static_cast<int64_t>(sizeof(T)) == kRowBytes;
  const bool k_adj = a.k_sh * static_cast<int64_t>(sizeof(T)) == kRowBytes;
  const bool v_adj = a.v_sh * static_cast<int64_t>(sizeof(T)) == kRowBytes;

  // positions / slots of tokens [meta_base, meta_base + 32), lane j holding token meta_base + j
  const int t_stop = (n_begin + n_count - 1) / per_token + 1;  // past this warp's last token
  int meta_base = -64, my_pos = -1, my_slot = -1;
  auto load_meta = [&](int tb) {  // warp-uniform
    meta_base = tb;
    const int t = tb + lane;
    my_pos = -1;
    my_slot = -1;
    if (t < t_stop) {
      int64_t pos = load_index(a.positions, t) + a.position_offset;
      int64_t slot = a.slots[t];
      if (pos < 0 || pos >= a.max_position) {  // the token is not written at all
        raise_device_error(a.error_flag, PKV_DEVERR_BAD_SEQUENCE_LENGTH);
        pos = -1;
      } else if (slot >= a.num_slots) {  // its query rows are written, its key/value rows are not
        raise_device_error(a.error_flag, PKV_DEVERR_SLOT_OUT_OF_RANGE);
        slot = -1;
      }
      my_pos = static_cast<int>(pos);
      my_slot = slot < 0 ? -1 : static_cast<int>(slot);  // negative: a padding token (no key/value rows)
    }
  };

  // issue side: group (it_t, it_g) goes to stage it_s
  const int t0 = n_begin / per_token;
  const int g0 = n_begin - t0 * per_token;
  int it_n = 0, it_t = t0, it_g = g0, it_s = 0;
  auto issue = [&]() {  // warp-uniform
    if (it_n >= n_count) return;
    if (it_t - meta_base >= 32) load_meta(it_t);
    const int j = it_t - meta_base;
    const int pos = __shfl_sync(0xffffffffu, my_pos, j), slot = __shfl_sync(0xffffffffu, my_slot, j);
    if (lane == 0) {
      uint8_t* st = ring + it_s * stage_bytes;
      int* hdr = reinterpret_cast<int*>(st + R * kRowBytes + table_bytes);
      hdr[0] = pos;
      hdr[1] = slot;
      const int row0 = it_g * R, row1 = row0 + R < rows ? row0 + R : rows;
      const int qa = row0, qb = row1 < hq ? row1 : hq;
      const int ka = row0 > hq ? row0 : hq, kb = row1 < hq + hkv ? row1 : hq + hkv;
      const int va = row0 > hq + hkv ? row0 : hq + hkv, vb = row1;
      const int nq = qb - qa > 0 ? qb - qa : 0;
      const int nk = slot >= 0 && kb - ka > 0 ? kb - ka : 0;
      const int nv = slot >= 0 && vb - va > 0 ? vb - va : 0;
      const bool table = a.rotary_dim > 0 && nq + nk > 0;
      const uint32_t bytes = pos < 0 ? 0u : static_cast<uint32_t>((nq + nk + nv) * kRowBytes + (table ? table_bytes : 0));
      fence_proxy_async_smem();  // the warp's reads of this stage's previous group come first
      mbar_arrive_expect_tx(&bars[it_s], bytes);
      if (pos >= 0) {
        const int64_t t = it_t;
        stage_rows<T, kRowBytes>(st, static_cast<const T*>(a.q) + t * a.q_st + qa * a.q_sh, nq, a.q_sh, q_adj,
                                 &bars[it_s]);
        stage_rows<T, kRowBytes>(st + (ka - row0) * kRowBytes,
                                 static_cast<const T*>(a.k) + t * a.k_st + (ka - hq) * a.k_sh, nk, a.k_sh, k_adj,
                                 &bars[it_s]);
        stage_rows<T, kRowBytes>(st + (va - row0) * kRowBytes,
                                 static_cast<const T*>(a.v) + t * a.v_st + (va - hq - hkv) * a.v_sh, nv, a.v_sh,
                                 v_adj, &bars[it_s]);
        if (table) {
          bulk_load(st + R * kRowBytes,
                    static_cast<const uint8_t*>(a.cos_sin) + static_cast<int64_t>(pos) * table_bytes, table_bytes,
                    &bars[it_s]);
        }
      }
    }
    ++it_n;
    if (++it_g == per_token) {
      it_g = 0;
      ++it_t;
    }
    if (++it_s == kNrStages) it_s = 0;
  };

  // The norm + rotary of this half's row `srow` (shared memory), stored at `out` when `store`. All lanes
  // of the warp call it together (shuffles).
  // srow / w1row / cs_s: shared-window addresses of the row, its (1 + w) table and the cos/sin row;
  // srow_g: the row as a generic pointer (only the shared-memory rotary uses it)
  auto norm_rope_rows = [&](uint32_t srow, T* srow_g, uint32_t w1row, T* out, bool store, uint32_t cs_s,
                            const T* cs_row) {
    // rms_norm -- squares rounded to fp32 then summed, as x.float().pow(2).mean() does,
    // x * (1 / sqrt(mean + eps)) * (1 + w) rounded to dtype
    uint32_t pw[CPL][WPC];
#pragma unroll
    for (int j = 0; j < CPL; ++j) lds_at<CB>(srow + (sl + LPR * j) * CB, pw[j]);
    // the run as fp32 pairs (elements 2 m, 2 m + 1 of the lane's run in pair m)
    constexpr int PPC = CE / 2;  // pairs per chunk
    uint64_t x2[EPL / 2];
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
#pragma unroll
      for (int m = 0; m < PPC; ++m) {
        if constexpr (sizeof(T) == 4) {
          x2[j * PPC + m] = f2_pack(__uint_as_float(pw[j][2 * m]), __uint_as_float(pw[j][2 * m + 1]));
        } else {
          x2[j * PPC + m] = widen2<T>(pw[j][m]);
        }
      }
    }
    uint64_t ss2 = f2_pack(0.f, 0.f);
#pragma unroll
    for (int m = 0; m < EPL / 2; ++m) ss2 = f2_add(ss2, f2_mul(x2[m], x2[m]));
    const float2 ssp = f2_unpack(ss2);
    float ss = __fadd_rn(ssp.x, ssp.y);
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = 1.f / sqrtf(ss / static_cast<float>(D) + a.eps);
    const uint64_t inv2 = f2_pack(inv, inv);
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
#pragma unroll
      for (int i = 0; i < CE; i += kW) {
        const uint32_t wr = w1row + ((j * (CE / kW) + i / kW) * LPR + sl) * kW * 4;
        if constexpr (kW == 4) {
          uint64_t w0, w1v;
          lds_pairs2(wr, w0, w1v);
          x2[j * PPC + i / 2] = f2_mul(f2_mul(x2[j * PPC + i / 2], inv2), w0);
          x2[j * PPC + i / 2 + 1] = f2_mul(f2_mul(x2[j * PPC + i / 2 + 1], inv2), w1v);
        } else {
          x2[j * PPC + i / 2] = f2_mul(f2_mul(x2[j * PPC + i / 2], inv2), lds_pair(wr));
        }
      }
    }
    // rounded to dtype, back into the chunk words
#pragma unroll
    for (int j = 0; j < CPL; ++j) {
#pragma unroll
      for (int m = 0; m < PPC; ++m) {
        if constexpr (sizeof(T) == 4) {
          const float2 f = f2_unpack(x2[j * PPC + m]);
          pw[j][2 * m] = __float_as_uint(f.x);
          pw[j][2 * m + 1] = __float_as_uint(f.y);
        } else {
          pw[j][m] = narrow2<T>(x2[j * PPC + m]);
        }
      }
    }
    // rotary: x_p' = rnd(rnd(x_p cos_p) + rnd(-x_q sin_p)), x_q' = rnd(rnd(x_q cos_q) + rnd(x_p sin_q)),
    // q = p + r / 2, products and sums rounded separately (never fused)
    if (rot_in_regs) {
      const bool lower = sl < dc;
      uint32_t cos_w[WPC] = {}, sin_w[WPC] = {};
      if (sl < rot_lanes) {
        lds_at<CB>(cs_s + sl * CB, cos_w);
        lds_at<CB>(cs_s + r * static_cast<int>(sizeof(T)) + sl * CB, sin_w);
      }
#pragma unroll
      for (int w = 0; w < WPC; ++w) {
        const uint32_t pv = __shfl_sync(0xffffffffu, pw[0][w], partner);
        if (sl < rot_lanes) {
          if constexpr (sizeof(T) == 4) {
            const float pf = lower ? -__uint_as_float(pv) : __uint_as_float(pv);
            pw[0][w] = __float_as_uint(__fadd_rn(__fmul_rn(__uint_as_float(pw[0][w]), __uint_as_float(cos_w[w])),
                                                 __fmul_rn(pf, __uint_as_float(sin_w[w]))));
          } else {
            const uint32_t pn = lower ? pv ^ 0x80008000u : pv;
            pw[0][w] = add2_rn<T>(mul2_rn<T>(pw[0][w], cos_w[w]), mul2_rn<T>(pn, sin_w[w]));
          }
        }
      }
    } else if (r > 0) {
      // general rotary widths: the rounded row back into shared memory, one (p, q) pair per lane at a time
#pragma unroll
      for (int j = 0; j < CPL; ++j) st_words<CB>(srow_g + (sl + LPR * j) * CE, pw[j]);
      __syncwarp();
      T* srow = srow_g;
      for (int p = sl; p < r / 2; p += LPR) {
        const int q = p + r / 2;
        const float xp = Elem<T>::to_f(srow[p]), xq = Elem<T>::to_f(srow[q]);
        const float cp = Elem<T>::to_f(cs_row[p]), cq = Elem<T>::to_f(cs_row[q]);
        const float sp = Elem<T>::to_f(cs_row[r + p]), sq = Elem<T>::to_f(cs_row[r + q]);
        const T m0 = Elem<T>::from_f(__fmul_rn(xp, cp)), m1 = Elem<T>::from_f(__fmul_rn(-xq, sp));
        const T m2 = Elem<T>::from_f(__fmul_rn(xq, cq)), m3 = Elem<T>::from_f(__fmul_rn(xp, sq));
        srow[p] = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(m0), Elem<T>::to_f(m1)));
        srow[q] = Elem<T>::from_f(__fadd_rn(Elem<T>::to_f(m2), Elem<T>::to_f(m3)));
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < CPL; ++j) lds_words<CB>(srow_g + (sl + LPR * j) * CE, pw[j]);
    }
    if (store) {
#pragma unroll
      for (int j = 0; j < CPL; ++j) st_words<CB>(out + (sl + LPR * j) * CE, pw[j]);
    }
  };

#pragma unroll
  for (int s = 0; s < kNrStages - 1; ++s) issue();
  int ct = t0, cg = g0, cs = 0;
  uint32_t parity = 0;
  for (int n = 0; n < n_count; ++n) {
    issue();
    const bool ok = mbar_wait_bounded(&bars[cs], parity, kNrWaitNs);
    if (!__all_sync(0xffffffffu, ok)) {
      if (lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
      break;
    }
    uint8_t* st = ring + cs * stage_bytes;
    const int* hdr = reinterpret_cast<const int*>(st + R * kRowBytes + table_bytes);
    const int pos = hdr[0], slot = hdr[1];
    if (pos >= 0) {
      const int row0 = cg * R, row1 = row0 + R < rows ? row0 + R : rows;
      const int qb = row1 < hq ? row1 : hq;
      const int ka = row0 > hq ? row0 : hq, kb = row1 < hq + hkv ? row1 : hq + hkv;
      const int va = row0 > hq + hkv ? row0 : hq + hkv;
      const T* cs_row = reinterpret_cast<const T*>(st + R * kRowBytes);
      const uint32_t st_s = smem_u32(st), cs_s = st_s + R * kRowBytes, w1_s = smem_u32(w1);
      T* q_tok = static_cast<T*>(a.q_out) + static_cast<int64_t>(ct) * a.qo_st;
#pragma unroll 1
      for (int row = row0; row < qb; row += RPS) {
        const int mine = row + half < qb ? row + half : row;  // an odd last row: the other half repeats it
        norm_rope_rows(st_s + (mine - row0) * kRowBytes, reinterpret_cast<T*>(st + (mine - row0) * kRowBytes), w1_s,
                       q_tok + mine * a.qo_sh, row + half < qb, cs_s, cs_row);
      }
      if (slot >= 0) {
        const int page = a.bs_shift >= 0 ? (slot >> a.bs_shift) : slot / static_cast<int>(a.block_size);
        const int64_t kv_off = static_cast<int64_t>(page) * a.sp + (slot - page * a.block_size) * a.ss;
        T* k_tok = static_cast<T*>(a.key_pool) + kv_off;
#pragma unroll 1
        for (int row = ka; row < kb; row += RPS) {
          const int mine = row + half < kb ? row + half : row;
          norm_rope_rows(st_s + (mine - row0) * kRowBytes, reinterpret_cast<T*>(st + (mine - row0) * kRowBytes),
                         w1_s + D * 4, k_tok + (mine - hq) * a.sh, row + half < kb, cs_s, cs_row);
        }
        T* v_tok = static_cast<T*>(a.value_pool) + kv_off;
#pragma unroll 1
        for (int row = va + half; row < row1; row += RPS) {  // value rows: copied as they are
          const uint32_t srow = st_s + (row - row0) * kRowBytes;
          T* out = v_tok + (row - hq - hkv) * a.sh;
#pragma unroll
          for (int j = 0; j < CPL; ++j) {
            uint32_t w[WPC];
            lds_at<CB>(srow + (sl + LPR * j) * CB, w);
            st_words<CB>(out + (sl + LPR * j) * CE, w);
          }
        }
      }
    }
    __syncwarp();  // every lane is done with this stage before a later issue refills it
    if (++cg == per_token) {
      cg = 0;
      ++ct;
    }
    if (++cs == kNrStages) {
      cs = 0;
      parity ^= 1u;
    }
  }
}

template <typename T, typename I, int EPL, int LPR>
int launch_nr(const RopeArgs<I>& a, int sms, cudaStream_t stream) {
  using Cfg = NrConfig<T, EPL, LPR>;
  auto kern = norm_rope_append_kernel<T, I, EPL, LPR>;
  const int table_bytes = 2 * a.rotary_dim * static_cast<int>(sizeof(T));
  const int smem = 2 * Cfg::kRowElems * 4 + kNrWarps * kNrBarBytes +
                   kNrWarps * kNrStages * (Cfg::kRows * Cfg::kRowBytes + table_bytes + 16);
  const cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return cuda_status(e, "norm_rope_append_kernel smem attribute");
  const int64_t per_token = (a.num_q_heads + 2 * a.num_kv_heads + Cfg::kRows - 1) / Cfg::kRows;
  const int64_t groups = a.num_tokens * per_token;
  const int64_t want = (groups + kNrWarps - 1) / kNrWarps;
  const int64_t per_sm = (227 * 1024) / (smem + 1024);
  const int64_t cap = static_cast<int64_t>(sms) * (per_sm > 0 ? per_sm : 1);
  const unsigned grid = static_cast<unsigned>(want < cap ? want : cap);
  kern<<<grid, kNrWarps * 32, smem, stream>>>(a);
  return cuda_status(cudaGetLastError(), "norm_rope_append_kernel launch");
}

template <typename T, typename I>
int launch_norm_rope(const RopeArgs<I>& a, int64_t head_dim, cudaStream_t stream) {
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  switch (head_dim) {
    case 64: return launch_nr<T, I, 4, 16>(a, sms, stream);
    case 128: return launch_nr<T, I, 8, 16>(a, sms, stream);
    case 256: return launch_nr<T, I, 16, 16>(a, sms, stream);
    case 512: return launch_nr<T, I, 16, 32>(a, sms, stream);
    default: return launch_nr<T, I, 32, 32>(a, sms, stream);
  }
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_qk_norm_rope_append(
    const void* query, int64_t q_stride_token, int64_t q_stride_head, const void* key, int64_t k_stride_token,
    int64_t k_stride_head, const void* value, int64_t v_stride_token, int64_t v_stride_head, const void* q_weight,
    const void* k_weight, float eps, const void* cos_sin, int64_t max_position, int64_t rotary_dim,
    const void* positions, int64_t position_offset, int index_dtype, const int64_t* slot_mapping, void* key_pool,
    void* value_pool, int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
    int64_t stride_page, int64_t stride_head, int64_t stride_slot, void* q_out, int64_t qo_stride_token,
    int64_t qo_stride_head, int64_t num_tokens, int64_t num_q_heads, int dtype, int32_t* error_flag, void* stream) {
  clear_error();
  const int es = dtype_size(dtype);
  PKV_REQUIRE(es > 0, "qk_norm_rope_append: unsupported dtype %d", dtype);
  PKV_REQUIRE(index_dtype == PKV_INDEX_I32 || index_dtype == PKV_INDEX_I64, "qk_norm_rope_append: bad index dtype");
  PKV_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512 || head_dim == 1024,
              "qk_norm_rope_append: head_dim must be 64, 128, 256, 512 or 1024 (got %lld)",
              static_cast<long long>(head_dim));
  const int64_t epl = head_dim / 32;
  PKV_REQUIRE(rotary_dim >= 0 && rotary_dim <= head_dim && rotary_dim % (2 * epl) == 0,
              "qk_norm_rope_append: rotary_dim must be a multiple of %lld in [0, head_dim]",
              static_cast<long long>(2 * epl));
  PKV_REQUIRE(num_tokens >= 0 && num_q_heads >= 0 && num_kv_heads > 0 && num_pages > 0 && block_size > 0,
              "qk_norm_rope_append: bad sizes");
  PKV_REQUIRE(num_q_heads + num_kv_heads < (1ll << 30), "qk_norm_rope_append: too many heads");
  PKV_REQUIRE(max_position > 0 && max_position < (1ll << 31), "qk_norm_rope_append: max_position must be in [1, 2^31)");
  PKV_REQUIRE(num_pages * block_size < (1ll << 31) && num_tokens * (num_q_heads + 2 * num_kv_heads) < (1ll << 31),
              "qk_norm_rope_append: pool slots and token rows must each stay below 2^31");
  PKV_REQUIRE(std::isfinite(eps) && eps >= 0.f, "qk_norm_rope_append: eps must be finite and non-negative");
  if (num_tokens == 0) return PKV_OK;
  PKV_REQUIRE(key && value && q_weight && k_weight && positions && slot_mapping && key_pool && value_pool,
              "qk_norm_rope_append: null pointer argument");
  PKV_REQUIRE(num_q_heads == 0 || (query && q_out), "qk_norm_rope_append: null query or q_out");
  PKV_REQUIRE(rotary_dim == 0 || cos_sin, "qk_norm_rope_append: null cos_sin table");
  // rows are streamed with 16-byte copies and each lane's run of head_dim / 32 elements is accessed as
  // a unit: row starts (pointers, strides) must be 16-byte aligned, table rows too
  const int64_t run = 16;
  const int64_t run_el = run / es;
  const uintptr_t ptrs = reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(key) |
                         reinterpret_cast<uintptr_t>(value) | reinterpret_cast<uintptr_t>(q_weight) |
                         reinterpret_cast<uintptr_t>(k_weight) | reinterpret_cast<uintptr_t>(cos_sin) |
                         reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool) |
                         reinterpret_cast<uintptr_t>(q_out);
  const int64_t strides[] = {q_stride_token, q_stride_head, k_stride_token, k_stride_head, v_stride_token,
                             v_stride_head, stride_page, stride_head, stride_slot, qo_stride_token, qo_stride_head,
                             rotary_dim};
  bool aligned = ptrs % static_cast<uintptr_t>(run) == 0;
  for (int64_t s : strides) aligned = aligned && s % run_el == 0;
  PKV_REQUIRE(aligned, "qk_norm_rope_append: pointers and strides must be aligned to %lld bytes",
              static_cast<long long>(run));
  bump_stat(kStatNormRopeAppend);
  const int32_t bs_shift = (block_size & (block_size - 1)) == 0 ? __builtin_ctzll(static_cast<uint64_t>(block_size)) : -1;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run_t = [&](auto tag, auto itag) -> int {
    using T = decltype(tag);
    using I = decltype(itag);
    RopeArgs<I> a{query,        q_stride_token, q_stride_head, key,        k_stride_token,
                  k_stride_head, value,         v_stride_token, v_stride_head, q_weight,
                  k_weight,      eps,           cos_sin,        max_position, static_cast<int32_t>(rotary_dim),
                  static_cast<const I*>(positions), position_offset, slot_mapping, key_pool, value_pool,
                  num_pages * block_size, block_size, stride_page, stride_head, stride_slot, bs_shift,
                  q_out,         qo_stride_token, qo_stride_head, num_tokens, static_cast<int32_t>(num_q_heads),
                  static_cast<int32_t>(num_kv_heads), error_flag};
    return launch_norm_rope<T, I>(a, head_dim, s);
  };
  auto run_i = [&](auto tag) -> int {
    if (index_dtype == PKV_INDEX_I32) return run_t(tag, int32_t{});
    return run_t(tag, int64_t{});
  };
  if (dtype == PKV_DTYPE_F32) return run_i(float{});
  if (dtype == PKV_DTYPE_F16) return run_i(__half{});
  return run_i(__nv_bfloat16{});
}
