// Fused q/k RMSNorm + partial rotary embedding + K/V append (the per-layer step in front of paged
// attention).
//
// The reference runs, per full-attention layer (src/tp_runtime.py:510-525, batched decode :2461-2483):
//   query = rms_norm(query, q_norm); key = rms_norm(key, k_norm)            (src/reference_ops.py:166-169)
//   cos, sin = rotary_embeddings(positions)                                 (src/reference_ops.py:203-212)
//   query, key = apply_rotary_pos_emb(query, key, cos, sin)                 (src/reference_ops.py:215-224)
//   key, value = _repeat_kv(...)[TP slice]; cache.append_blocks(key, value) (src/decode_state.py:271-293)
// as separate torch launches with the new K/V round-tripping through memory. Here one launch does it
// all: one warp per (token, head row); rows 0 .. Hq-1 are query heads (written to q_out), rows
// Hq .. Hq+Hkv-1 are the pool's KV heads (post-RoPE key and the raw value written straight into the
// token's slot; no repeated heads). Each lane holds D/32 consecutive elements of the row.
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

// Rounds a pair of fp32 values to the dtype (round to nearest even) and back to fp32, with one paired
// conversion instruction.
template <typename T>
__device__ __forceinline__ void rnd2(float& a, float& b);
template <>
__device__ __forceinline__ void rnd2<float>(float&, float&) {}
template <>
__device__ __forceinline__ void rnd2<__nv_bfloat16>(float& a, float& b) {
  const float2 f = __bfloat1622float2(__floats2bfloat162_rn(a, b));
  a = f.x;
  b = f.y;
}
template <>
__device__ __forceinline__ void rnd2<__half>(float& a, float& b) {
  const float2 f = __half22float2(__floats2half2_rn(a, b));
  a = f.x;
  b = f.y;
}

// Loads / stores N consecutive elements (N * sizeof(T) bytes, aligned to that size up to 16).
template <typename T, int N>
__device__ __forceinline__ void load_row(const T* p, float (&v)[N]) {
  constexpr int kBytes = N * static_cast<int>(sizeof(T));
  if constexpr (kBytes % 16 == 0) {
#pragma unroll
    for (int c = 0; c < kBytes / 16; ++c) {
      const uint4 w = reinterpret_cast<const uint4*>(p)[c];
      const T* e = reinterpret_cast<const T*>(&w);
#pragma unroll
      for (int i = 0; i < 16 / static_cast<int>(sizeof(T)); ++i) v[c * (16 / sizeof(T)) + i] = Elem<T>::to_f(e[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = Elem<T>::to_f(p[i]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_row(T* p, const float (&v)[N]) {
  constexpr int kBytes = N * static_cast<int>(sizeof(T));
  if constexpr (sizeof(T) == 2 && kBytes % 16 == 0) {  // paired conversions, 16-byte stores
#pragma unroll
    for (int c = 0; c < kBytes / 16; ++c)
      reinterpret_cast<uint4*>(p)[c] = make_uint4(pack2<T>(v[8 * c], v[8 * c + 1]), pack2<T>(v[8 * c + 2], v[8 * c + 3]),
                                                  pack2<T>(v[8 * c + 4], v[8 * c + 5]), pack2<T>(v[8 * c + 6], v[8 * c + 7]));
  } else if constexpr (kBytes % 16 == 0) {
#pragma unroll
    for (int c = 0; c < kBytes / 16; ++c) {
      uint4 w;
      T* e = reinterpret_cast<T*>(&w);
#pragma unroll
      for (int i = 0; i < 16 / static_cast<int>(sizeof(T)); ++i) e[i] = Elem<T>::from_f(v[c * (16 / sizeof(T)) + i]);
      reinterpret_cast<uint4*>(p)[c] = w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = Elem<T>::from_f(v[i]);
  }
}

// Stores N consecutive values that are already exact in the dtype (bf16: the high halves of the fp32
// patterns, one byte-permute per pair).
template <typename T, int N>
__device__ __forceinline__ void store_exact(T* p, const float (&v)[N]) {
  if constexpr (sizeof(T) == 4) {
    store_row<T, N>(p, v);
  } else {
    uint32_t w[N / 2];
#pragma unroll
    for (int i = 0; i < N / 2; ++i) {
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        w[i] = __byte_perm(__float_as_uint(v[2 * i]), __float_as_uint(v[2 * i + 1]), 0x7632);
      } else {
        const __half2 h = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    constexpr int kBytes = N * 2;
    if constexpr (kBytes % 16 == 0) {
#pragma unroll
      for (int c = 0; c < kBytes / 16; ++c)
        reinterpret_cast<uint4*>(p)[c] = make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
    } else if constexpr (kBytes % 8 == 0) {
#pragma unroll
      for (int c = 0; c < kBytes / 8; ++c) reinterpret_cast<uint2*>(p)[c] = make_uint2(w[2 * c], w[2 * c + 1]);
    } else {
#pragma unroll
      for (int c = 0; c < kBytes / 4; ++c) reinterpret_cast<uint32_t*>(p)[c] = w[c];
    }
  }
}

// N consecutive elements kept packed (as loaded) until they are processed.
template <typename T, int N>
struct RawRow {
  static constexpr int kWords = (N * static_cast<int>(sizeof(T)) + 3) / 4;
  uint32_t w[kWords];
};

template <typename T, int N>
__device__ __forceinline__ void load_raw(const T* p, RawRow<T, N>& r) {
  constexpr int kBytes = N * static_cast<int>(sizeof(T));
  if constexpr (kBytes % 16 == 0) {
#pragma unroll
    for (int c = 0; c < kBytes / 16; ++c) {
      const uint4 v = reinterpret_cast<const uint4*>(p)[c];
      r.w[4 * c] = v.x;
      r.w[4 * c + 1] = v.y;
      r.w[4 * c + 2] = v.z;
      r.w[4 * c + 3] = v.w;
    }
  } else if constexpr (kBytes % 8 == 0) {
#pragma unroll
    for (int c = 0; c < kBytes / 8; ++c) {
      const uint2 v = reinterpret_cast<const uint2*>(p)[c];
      r.w[2 * c] = v.x;
      r.w[2 * c + 1] = v.y;
    }
  } else {
    static_assert(kBytes % 4 == 0, "rows are at least 4-byte runs");
#pragma unroll
    for (int c = 0; c < kBytes / 4; ++c) r.w[c] = reinterpret_cast<const uint32_t*>(p)[c];
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_raw(T* p, const RawRow<T, N>& r) {
  constexpr int kBytes = N * static_cast<int>(sizeof(T));
  if constexpr (kBytes % 16 == 0) {
#pragma unroll
    for (int c = 0; c < kBytes / 16; ++c)
      reinterpret_cast<uint4*>(p)[c] = make_uint4(r.w[4 * c], r.w[4 * c + 1], r.w[4 * c + 2], r.w[4 * c + 3]);
  } else if constexpr (kBytes % 8 == 0) {
#pragma unroll
    for (int c = 0; c < kBytes / 8; ++c) reinterpret_cast<uint2*>(p)[c] = make_uint2(r.w[2 * c], r.w[2 * c + 1]);
  } else {
#pragma unroll
    for (int c = 0; c < kBytes / 4; ++c) reinterpret_cast<uint32_t*>(p)[c] = r.w[c];
  }
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
  void* q_out;
  int64_t qo_st, qo_sh;
  int64_t num_tokens;
  int32_t num_q_heads, num_kv_heads;
  int32_t* error_flag;
};

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gmem_src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

constexpr int kNrWarps = 4;   // warps per block
constexpr int kNrStages = 3;  // row groups per warp: one being processed, two in flight

template <typename T, int EPL>
struct NrConfig {
  static constexpr int kRowBytes = 32 * EPL * static_cast<int>(sizeof(T));
  static constexpr int kRows = kRowBytes >= 2048 ? 1 : 2048 / kRowBytes;  // items per group
};

// Items are (token, row) with rows = Hq query rows, Hkv key rows, Hkv value rows of the token. A group is
// up to kRows consecutive rows of ONE token (a token spans ceil(rows / kRows) groups), so its position,
// slot and cos/sin row are looked up once. Each warp takes groups grid-stride and stages each in a
// private kNrStages-deep ring of shared memory, two groups ahead of the one it processes: lane 0 loads
// the token's position and slot, then 16-byte cp.async copies bring the input rows and the token's
// cos/sin row. Processing reads only shared memory: query/key rows are normalised and rotated, value
// rows copied. No registers hold rows in flight.
// Stage layout: kRows input rows | one cos/sin row (2 * rotary_dim elements) | {position, slot}.
template <typename T, typename I, int EPL>
__global__ void __launch_bounds__(kNrWarps * 32) norm_rope_append_kernel(const RopeArgs<I> a) {
  using Cfg = NrConfig<T, EPL>;
  constexpr int R = Cfg::kRows;
  constexpr int kChunks = Cfg::kRowBytes / 16;  // a power of two
  extern __shared__ __align__(16) uint8_t nr_smem[];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int table_bytes = 2 * a.rotary_dim * static_cast<int>(sizeof(T));
  const int stage_bytes = R * Cfg::kRowBytes + table_bytes + 16;
  uint8_t* ring = nr_smem + warp * (kNrStages * stage_bytes);
  const int rows = a.num_q_heads + 2 * a.num_kv_heads;
  const int per_token = (rows + R - 1) / R;  // groups per token
  const int64_t groups = a.num_tokens * per_token;
  const int64_t gw = static_cast<int64_t>(blockIdx.x) * kNrWarps + warp;
  const int64_t nw = static_cast<int64_t>(gridDim.x) * kNrWarps;
  float wq[EPL], wk[EPL];
  load_row<T, EPL>(static_cast<const T*>(a.q_weight) + lane * EPL, wq);
  load_row<T, EPL>(static_cast<const T*>(a.k_weight) + lane * EPL, wk);
  const int half = a.rotary_dim >> 1;
  const int first = lane * EPL;

  // Stages group g (if it exists) into `stage`; always commits one cp.async group so that the wait
  // counts stay uniform.
  auto issue = [&](int64_t g, int stage) {
    if (g < groups) {
      // groups < 2^31 (checked on the host): 32-bit division
      const int64_t t = static_cast<uint32_t>(g) / static_cast<uint32_t>(per_token);
      const int row0 = static_cast<int>(g - t * per_token) * R;
      uint8_t* st = ring + stage * stage_bytes;
      int64_t pos = 0;
      if (lane == 0) {
        pos = load_index(a.positions, t) + a.position_offset;
        int64_t slot = row0 + R > a.num_q_heads ? a.slots[t] : 0;  // the group holds key/value rows
        if (pos < 0 || pos >= a.max_position) {  // the token is not written at all
          if (row0 == 0) raise_device_error(a.error_flag, PKV_DEVERR_BAD_SEQUENCE_LENGTH);
          pos = -1;
        } else if (slot >= a.num_slots) {
          if (row0 <= a.num_q_heads && a.num_q_heads < row0 + R)
            raise_device_error(a.error_flag, PKV_DEVERR_SLOT_OUT_OF_RANGE);
          slot = -1;
        }
        reinterpret_cast<int64_t*>(st + R * Cfg::kRowBytes + table_bytes)[0] = pos;
        reinterpret_cast<int64_t*>(st + R * Cfg::kRowBytes + table_bytes)[1] = slot;
      }
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        if (row >= rows) break;
        const T* src;
        if (row < a.num_q_heads) {
          src = static_cast<const T*>(a.q) + t * a.q_st + static_cast<int64_t>(row) * a.q_sh;
        } else if (row < a.num_q_heads + a.num_kv_heads) {
          src = static_cast<const T*>(a.k) + t * a.k_st + static_cast<int64_t>(row - a.num_q_heads) * a.k_sh;
        } else {
          src = static_cast<const T*>(a.v) + t * a.v_st +
                static_cast<int64_t>(row - a.num_q_heads - a.num_kv_heads) * a.v_sh;
        }
        const uint8_t* src_b = reinterpret_cast<const uint8_t*>(src);
        uint8_t* dst_b = st + r * Cfg::kRowBytes;
#pragma unroll
        for (int c = lane; c < kChunks; c += 32) cp_async16(dst_b + c * 16, src_b + c * 16);
      }
      pos = __shfl_sync(0xffffffffu, pos, 0);
      if (pos >= 0 && row0 < a.num_q_heads + a.num_kv_heads) {  // query or key rows: their cos/sin row
        const uint8_t* src = reinterpret_cast<const uint8_t*>(a.cos_sin) + pos * table_bytes;
        for (int c = lane; c < table_bytes / 16; c += 32) cp_async16(st + R * Cfg::kRowBytes + c * 16, src + c * 16);
      }
    }
    cp_async_commit();
  };

#pragma unroll
  for (int s = 0; s < kNrStages - 1; ++s) issue(gw + s * nw, s);
  for (int64_t k = 0;; ++k) {
    const int64_t g = gw + k * nw;
    if (g >= groups) break;
    issue(gw + (k + kNrStages - 1) * nw, static_cast<int>((k + kNrStages - 1) % kNrStages));
    cp_async_wait<kNrStages - 1>();  // this lane's copies of group g have landed
    __syncwarp();                    // ... and every other lane's, and the position / slot
    uint8_t* st = ring + static_cast<int>(k % kNrStages) * stage_bytes;
    const int64_t pos = reinterpret_cast<const int64_t*>(st + R * Cfg::kRowBytes + table_bytes)[0];
    const int64_t slot = reinterpret_cast<const int64_t*>(st + R * Cfg::kRowBytes + table_bytes)[1];
    const int64_t t = static_cast<uint32_t>(g) / static_cast<uint32_t>(per_token);
    const int row0 = static_cast<int>(g - t * per_token) * R;
    if (pos >= 0) {
      const T* cs = reinterpret_cast<const T*>(st + R * Cfg::kRowBytes);
      // slots < num_slots < 2^31 (checked on the host): 32-bit division
      const int64_t page = slot >= 0 ? static_cast<uint32_t>(slot) / static_cast<uint32_t>(a.block_size) : 0;
      const int64_t off = slot - page * a.block_size;
#pragma unroll 1
      for (int r = 0; r < R; ++r) {
        const int row = row0 + r;
        if (row >= rows) break;
        T* srow = reinterpret_cast<T*>(st + r * Cfg::kRowBytes);
        const int h = row - a.num_q_heads;
        if (h >= 0 && slot < 0) continue;  // key/value rows of a padding token (or a bad slot)
        T* out;
        if (h < 0) {
          out = static_cast<T*>(a.q_out) + t * a.qo_st + static_cast<int64_t>(row) * a.qo_sh;
        } else if (h < a.num_kv_heads) {
          out = static_cast<T*>(a.key_pool) + page * a.sp + static_cast<int64_t>(h) * a.sh + off * a.ss;
        } else {
          out = static_cast<T*>(a.value_pool) + page * a.sp + static_cast<int64_t>(h - a.num_kv_heads) * a.sh +
                off * a.ss;
        }
        if (h < a.num_kv_heads) {
          // phase 1 (all lanes, contiguous chunk): rms_norm in place -- squares rounded to fp32 then
          // summed, as x.float().pow(2).mean() does, x * (1 / sqrt(mean + eps)) * (1 + w) rounded to dtype
          float x[EPL];
          load_row<T, EPL>(srow + first, x);
          const float* w = h < 0 ? wq : wk;
          uint64_t ss2 = f2_pack(0.f, 0.f);
#pragma unroll
          for (int i = 0; i < EPL; i += 2) {
            const uint64_t xi = f2_pack(x[i], x[i + 1]);
            ss2 = f2_add(ss2, f2_mul(xi, xi));
          }
          const float2 ssp = f2_unpack(ss2);
          float ss = __fadd_rn(ssp.x, ssp.y);
#pragma unroll
          for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
          const float inv = 1.f / sqrtf(ss / static_cast<float>(32 * EPL) + a.eps);
          const uint64_t inv2 = f2_pack(inv, inv);
#pragma unroll
          for (int i = 0; i < EPL; i += 2) {
            const float2 y = f2_unpack(f2_mul(f2_mul(f2_pack(x[i], x[i + 1]), inv2), f2_pack(1.f + w[i], 1.f + w[i + 1])));
            x[i] = y.x;
            x[i + 1] = y.y;
          }
          store_row<T, EPL>(srow + first, x);  // rounds to dtype
          if (a.rotary_dim > 0) {
            __syncwarp();
            // phase 2 (all lanes, one (element, partner) pair each at a time): rotary in place,
            // x_p' = rnd(rnd(x_p cos_p) + rnd(-x_q sin_p)), x_q' = rnd(rnd(x_q cos_q) + rnd(x_p sin_q))
            // with q = p + rotary_dim / 2; products and sums rounded separately (never fused)
            for (int p = lane; p < half; p += 32) {
              const int q = p + half;
              float xp = Elem<T>::to_f(srow[p]), xq = Elem<T>::to_f(srow[q]);
              const float cp = Elem<T>::to_f(cs[p]), cq = Elem<T>::to_f(cs[q]);
              const float sp = Elem<T>::to_f(cs[a.rotary_dim + p]), sq = Elem<T>::to_f(cs[a.rotary_dim + q]);
              float m0 = __fmul_rn(xp, cp), m1 = __fmul_rn(-xq, sp), m2 = __fmul_rn(xq, cq), m3 = __fmul_rn(xp, sq);
              rnd2<T>(m0, m1);
              rnd2<T>(m2, m3);
              float o0 = __fadd_rn(m0, m1), o1 = __fadd_rn(m2, m3);
              rnd2<T>(o0, o1);
              srow[p] = Elem<T>::from_f(o0);
              srow[q] = Elem<T>::from_f(o1);
            }
          }
          __syncwarp();
        }
        // phase 3 (all lanes): the row out, 16-byte runs
        RawRow<T, EPL> v;
        load_raw<T, EPL>(srow + first, v);
        store_raw<T, EPL>(out + first, v);
      }
    }
    __syncwarp();  // every lane is done with this stage before a later issue refills it
  }
  cp_async_wait<0>();  // prefetches past the last group were empty commits; nothing is left in flight
}

template <typename T, typename I, int EPL>
int launch_nr(const RopeArgs<I>& a, int sms, cudaStream_t stream) {
  using Cfg = NrConfig<T, EPL>;
  auto kern = norm_rope_append_kernel<T, I, EPL>;
  const int table_bytes = 2 * a.rotary_dim * static_cast<int>(sizeof(T));
  const int smem = kNrWarps * kNrStages * (Cfg::kRows * Cfg::kRowBytes + table_bytes + 16);
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
    case 64: return launch_nr<T, I, 2>(a, sms, stream);
    case 128: return launch_nr<T, I, 4>(a, sms, stream);
    case 256: return launch_nr<T, I, 8>(a, sms, stream);
    case 512: return launch_nr<T, I, 16>(a, sms, stream);
    default: return launch_nr<T, I, 32>(a, sms, stream);
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
  PKV_REQUIRE(max_position > 0, "qk_norm_rope_append: max_position must be positive");
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
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run_t = [&](auto tag, auto itag) -> int {
    using T = decltype(tag);
    using I = decltype(itag);
    RopeArgs<I> a{query,        q_stride_token, q_stride_head, key,        k_stride_token,
                  k_stride_head, value,         v_stride_token, v_stride_head, q_weight,
                  k_weight,      eps,           cos_sin,        max_position, static_cast<int32_t>(rotary_dim),
                  static_cast<const I*>(positions), position_offset, slot_mapping, key_pool, value_pool,
                  num_pages * block_size, block_size, stride_page, stride_head, stride_slot,
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
