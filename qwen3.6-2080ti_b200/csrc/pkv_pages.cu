// Byte-exact page movers: slot-mapped append, block-table gather and page copy/compaction.
//
// All three are HBM-bound copies. Every thread moves 16-byte vectors (falling back to 8/4/2 bytes
// when a pointer or stride is not aligned), grid-stride over all vectors of the call, with the K
// and V moves of one vector issued together for memory-level parallelism. Grids are sized as a
// multiple of the SM count.
#include <algorithm>

#include <type_traits>

#include "pkv_common.cuh"

namespace pkv {
namespace {

template <int VB>
struct VecT;
template <> struct VecT<16> { using type = uint4; };
template <> struct VecT<8> { using type = uint2; };
template <> struct VecT<4> { using type = uint32_t; };
template <> struct VecT<2> { using type = uint16_t; };

int g_num_sms = 0;

int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms = sms > 0 ? sms : 148;
  }
  return g_num_sms;
}

int64_t grid_for(int64_t work_items, int threads) {
  const int64_t cap = static_cast<int64_t>(num_sms()) * 16;
  return std::max<int64_t>(1, std::min<int64_t>(cap, ceil_div(work_items, threads)));
}

// Largest vector width (16/8/4/2 bytes) that divides every given byte quantity.
int vector_bytes(std::initializer_list<int64_t> quantities, int esize) {
  int vb = 16;
  for (int64_t q : quantities) {
    while (vb > esize && (q % vb) != 0) vb >>= 1;
  }
  return std::max(vb, esize);
}

// ---- a1: slot-mapped append -----------------------------------------------------------------------
struct AppendArgs {
  const char* key;
  const char* value;
  int64_t k_tok, k_head, v_tok, v_head;  // bytes
  const int64_t* slots;  // nullptr: slots from `table` for positions start, start + 1, ...
  const int64_t* table;
  int64_t table_len, start;
  int64_t num_tokens;
  char* kpool;
  char* vpool;
  int64_t num_slots;  // num_pages * block_size
  int64_t block_size;
  int64_t p_page, p_head, p_slot;  // bytes
  int64_t heads;
  int64_t vec_per_row;
  int32_t* error_flag;
};

template <int VB>
__global__ void __launch_bounds__(256) kv_append_kernel(AppendArgs a) {
  using V = typename VecT<VB>::type;
  const int64_t total = a.num_tokens * a.heads * a.vec_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = i / a.vec_per_row;
    const int64_t vec = i - row * a.vec_per_row;
    const int64_t token = row / a.heads;
    const int64_t head = row - token * a.heads;
    int64_t slot;
    if (a.slots != nullptr) {
      slot = a.slots[token];
      if (slot < 0) continue;  // padding token
    } else {
      const int64_t pos = a.start + token;
      const int64_t logical = pos / a.block_size;
      if (logical >= a.table_len) {
        if (vec == 0 && head == 0) raise_device_error(a.error_flag, PKV_DEVERR_TABLE_TOO_SHORT);
        continue;
      }
      const int64_t page = a.table[logical];
      if (page < 0 || page * a.block_size >= a.num_slots) {
        if (vec == 0 && head == 0) raise_device_error(a.error_flag, PKV_DEVERR_PAGE_OUT_OF_RANGE);
        continue;
      }
      slot = page * a.block_size + (pos - logical * a.block_size);
    }
    if (slot >= a.num_slots) {
      if (vec == 0) raise_device_error(a.error_flag, PKV_DEVERR_SLOT_OUT_OF_RANGE);
      continue;
    }
    const int64_t page = slot / a.block_size;
    const int64_t off = slot - page * a.block_size;
    const int64_t dst = page * a.p_page + head * a.p_head + off * a.p_slot + vec * VB;
    const V kv = *reinterpret_cast<const V*>(a.key + token * a.k_tok + head * a.k_head + vec * VB);
    const V vv = *reinterpret_cast<const V*>(a.value + token * a.v_tok + head * a.v_head + vec * VB);
    *reinterpret_cast<V*>(a.kpool + dst) = kv;
    *reinterpret_cast<V*>(a.vpool + dst) = vv;
  }
}

// ---- a1/a2: decode-step slot mapping ---------------------------------------------------------------
template <typename I>
__global__ void __launch_bounds__(256) decode_slots_kernel(const I* tables, int64_t table_stride, int64_t max_blocks,
                                                           I* seq_lens, int64_t batch, int64_t block_size,
                                                           int64_t num_pages, int64_t* slots, int advance,
                                                           int64_t layers, int32_t* error_flag) {
  const int64_t b = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x;
  if (b >= batch) return;
  const int64_t len = static_cast<int64_t>(seq_lens[b]);
  int64_t slot = -1;
  if (len >= 0) {
    const int64_t logical = len / block_size;
    if (logical >= max_blocks) {
      raise_device_error(error_flag, PKV_DEVERR_TABLE_TOO_SHORT);
    } else {
      const int64_t page = static_cast<int64_t>(tables[b * table_stride + logical]);
      if (page < 0 || page >= num_pages) {
        raise_device_error(error_flag, PKV_DEVERR_PAGE_OUT_OF_RANGE);
      } else {
        slot = page * block_size + (len - logical * block_size);
        if (advance) seq_lens[b] = static_cast<I>(len + 1);
      }
    }
  }
  // layer l's pool is pages [l * num_pages, (l + 1) * num_pages) of the layers' stacked pools
  for (int64_t l = 0; l < layers; ++l) slots[l * batch + b] = slot < 0 ? -1 : slot + l * num_pages * block_size;
}

// ---- a3: gather into dense logical order ------------------------------------------------------------
template <typename I>
struct GatherArgs {
  const char* kpool;
  const char* vpool;
  int64_t num_pages, block_size;
  int64_t p_page, p_head, p_slot;  // bytes
  const I* tables;
  int64_t table_stride, max_blocks;
  const I* seq_lens;
  int64_t batch, heads, max_len;
  char* kout;
  char* vout;
  int64_t o_b, o_h, o_t;  // bytes
  int64_t vec_per_row;
  int32_t* error_flag;
};

template <int VB, typename I>
__global__ void __launch_bounds__(256) kv_gather_kernel(GatherArgs<I> a) {
  using V = typename VecT<VB>::type;
  const int64_t total = a.batch * a.heads * a.max_len * a.vec_per_row;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    int64_t row = i / a.vec_per_row;
    const int64_t vec = i - row * a.vec_per_row;
    const int64_t pos = row % a.max_len;
    row /= a.max_len;
    const int64_t head = row % a.heads;
    const int64_t b = row / a.heads;
    const int64_t out = b * a.o_b + head * a.o_h + pos * a.o_t + vec * VB;
    V kv{}, vv{};
    const int64_t len = load_index(a.seq_lens, b);
    if (pos < len) {
      const int64_t logical = pos / a.block_size;
      const int64_t page = logical < a.max_blocks ? load_index(a.tables, b * a.table_stride + logical) : -1;
      if (page >= 0 && page < a.num_pages) {
        const int64_t src = page * a.p_page + head * a.p_head + (pos - logical * a.block_size) * a.p_slot + vec * VB;
        kv = *reinterpret_cast<const V*>(a.kpool + src);
        vv = *reinterpret_cast<const V*>(a.vpool + src);
      } else if (vec == 0) {
        raise_device_error(a.error_flag,
                           logical < a.max_blocks ? PKV_DEVERR_PAGE_OUT_OF_RANGE : PKV_DEVERR_TABLE_TOO_SHORT);
      }
    }
    *reinterpret_cast<V*>(a.kout + out) = kv;
    *reinterpret_cast<V*>(a.vout + out) = vv;
  }
}

// ---- a10: page copy ---------------------------------------------------------------------------------
struct CopyArgs {
  char* kpool;
  char* vpool;
  int64_t num_layers, layer_stride;
  int64_t num_pages, page_stride;
  int64_t chunks, chunk_stride;
  int64_t vec_per_chunk;
  const int32_t* src;
  const int32_t* dst;
  int64_t num_pairs;
  int32_t* error_flag;
};

// One work item = one vector of one chunk of one (layer, pair); both pools are moved by the same
// thread. Four items per thread are loaded before any is stored to keep more bytes in flight.
template <int VB>
__global__ void __launch_bounds__(256) copy_pages_kernel(CopyArgs a) {
  using V = typename VecT<VB>::type;
  constexpr int kUnroll = 4;
  const int64_t per_pair = a.chunks * a.vec_per_chunk;
  const int64_t total = a.num_layers * a.num_pairs * per_pair;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t base = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; base < total;
       base += stride * kUnroll) {
    V kbuf[kUnroll], vbuf[kUnroll];
    int64_t dst_off[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t i = base + u * stride;
      dst_off[u] = -1;
      if (i >= total) continue;
      int64_t rest = i;
      const int64_t vec = rest % a.vec_per_chunk;
      rest /= a.vec_per_chunk;
      const int64_t chunk = rest % a.chunks;
      rest /= a.chunks;
      const int64_t pair = rest % a.num_pairs;
      const int64_t layer = rest / a.num_pairs;
      const int64_t s = a.src[pair];
      const int64_t d = a.dst[pair];
      if (s < 0 || s >= a.num_pages || d < 0 || d >= a.num_pages) {
        if (vec == 0 && chunk == 0 && layer == 0) raise_device_error(a.error_flag, PKV_DEVERR_PAGE_OUT_OF_RANGE);
        continue;
      }
      const int64_t common = layer * a.layer_stride + chunk * a.chunk_stride + vec * VB;
      const int64_t src_off = common + s * a.page_stride;
      dst_off[u] = common + d * a.page_stride;
      if (a.kpool) kbuf[u] = *reinterpret_cast<const V*>(a.kpool + src_off);
      if (a.vpool) vbuf[u] = *reinterpret_cast<const V*>(a.vpool + src_off);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (dst_off[u] < 0) continue;
      if (a.kpool) *reinterpret_cast<V*>(a.kpool + dst_off[u]) = kbuf[u];
      if (a.vpool) *reinterpret_cast<V*>(a.vpool + dst_off[u]) = vbuf[u];
    }
  }
}


// ---- FP8 (e4m3) append: per-(slot, KV head) scales ---------------------------------------------------------
// Two fp32 values -> two e4m3 bytes (round to nearest even, saturating to +-448; NaN stays NaN), lo first.
__device__ __forceinline__ uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

template <typename T, int EPL>
struct Fp8AppendArgs {
  const T* key;
  const T* value;
  int64_t k_st, k_sh, v_st, v_sh;  // elements
  const int64_t* slots;
  int64_t num_tokens;
  uint8_t* key_pool;
  uint8_t* value_pool;
  float* k_scales;
  float* v_scales;
  int64_t num_slots, block_size, sp, sh, ss;  // pool strides in bytes (= elements)
  int64_t scale_sp, scale_sh;                  // floats; slot stride 1
  int32_t num_kv_heads;
  int32_t* error_flag;
};

// One warp per (token, KV head, K or V) row; lane l quantises elements [l * EPL, (l + 1) * EPL):
//   amax = max |x|, scale = amax / 448, code = e4m3(x * (448 / amax)) (zero rows: scale 0, codes 0),
// the row's codes go to its slot and the scale to the slot's entry of the scale pool.
template <typename T, int EPL>
__global__ void __launch_bounds__(256) kv_append_fp8_kernel(const Fp8AppendArgs<T, EPL> a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t rows = a.num_tokens * a.num_kv_heads * 2;
  for (int64_t item = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); item < rows;
       item += warps) {
    const int64_t t = item / (2 * a.num_kv_heads);
    const int rem = static_cast<int>(item - t * 2 * a.num_kv_heads);
    const int h = rem >> 1;
    const bool is_v = rem & 1;
    const int64_t slot = a.slots[t];
    if (slot < 0) continue;  // padding token
    if (slot >= a.num_slots) {
      if (lane == 0 && rem == 0) raise_device_error(a.error_flag, PKV_DEVERR_SLOT_OUT_OF_RANGE);
      continue;
    }
    const T* src = is_v ? a.value + t * a.v_st + h * a.v_sh : a.key + t * a.k_st + h * a.k_sh;
    float x[EPL];
#pragma unroll
    for (int i = 0; i < EPL; ++i) x[i] = Elem<T>::to_f(src[lane * EPL + i]);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) amax = fmaxf(amax, fabsf(x[i]));
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float inv = amax > 0.f ? __fdiv_rn(448.f, amax) : 0.f;
    const float scale = __fdiv_rn(amax, 448.f);
    const int64_t page = slot / a.block_size, off = slot - page * a.block_size;
    uint8_t* dst = (is_v ? a.value_pool : a.key_pool) + page * a.sp + h * a.sh + off * a.ss + lane * EPL;
    uint32_t words[(EPL + 3) / 4] = {};
#pragma unroll
    for (int i = 0; i < EPL; i += 2) {
      const uint32_t pair = f32x2_to_e4m3x2(__fmul_rn(x[i], inv), __fmul_rn(x[i + 1], inv));
      words[i / 4] |= pair << (8 * (i % 4));
    }
    if constexpr (EPL % 4 == 0) {
#pragma unroll
      for (int w = 0; w < EPL / 4; ++w) reinterpret_cast<uint32_t*>(dst)[w] = words[w];
    } else {
      *reinterpret_cast<uint16_t*>(dst) = static_cast<uint16_t>(words[0]);
    }
    if (lane == 0) (is_v ? a.v_scales : a.k_scales)[page * a.scale_sp + h * a.scale_sh + off] = scale;
  }
}

template <typename T, int EPL>
int launch_append_fp8(const Fp8AppendArgs<T, EPL>& a, cudaStream_t s) {
  const int64_t rows = a.num_tokens * a.num_kv_heads * 2;
  const int64_t grid = grid_for((rows + 7) / 8, 1);
  kv_append_fp8_kernel<T, EPL><<<grid, 256, 0, s>>>(a);
  return cuda_status(cudaGetLastError(), "kv_append_fp8 launch");
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_kv_append(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                             const void* value, int64_t value_stride_token, int64_t value_stride_head,
                             const int64_t* slot_mapping, int64_t num_tokens, void* key_pool, void* value_pool,
                             int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                             int64_t stride_page, int64_t stride_head, int64_t stride_slot, int dtype,
                             int32_t* error_flag, void* stream) {
  clear_error();
  const int es = dtype_size(dtype);
  PKV_REQUIRE(es > 0, "kv_append: unsupported dtype %d", dtype);
  PKV_REQUIRE(num_tokens >= 0, "kv_append: num_tokens must be non-negative");
  PKV_REQUIRE(num_kv_heads > 0 && head_dim > 0 && block_size > 0 && num_pages > 0,
              "kv_append: heads, head_dim, block_size and num_pages must be positive");
  if (num_tokens == 0) return PKV_OK;
  PKV_REQUIRE(key && value && slot_mapping && key_pool && value_pool, "kv_append: null pointer argument");
  const int64_t row_bytes = head_dim * es;
  const int vb = vector_bytes({row_bytes, key_stride_token * es, key_stride_head * es, value_stride_token * es,
                               value_stride_head * es, stride_page * es, stride_head * es, stride_slot * es,
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(key)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(value)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(key_pool)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(value_pool))},
                              es);
  AppendArgs a{static_cast<const char*>(key), static_cast<const char*>(value),
               key_stride_token * es, key_stride_head * es, value_stride_token * es, value_stride_head * es,
               slot_mapping, nullptr, 0, 0, num_tokens, static_cast<char*>(key_pool), static_cast<char*>(value_pool),
               num_pages * block_size, block_size, stride_page * es, stride_head * es, stride_slot * es,
               num_kv_heads, row_bytes / vb, error_flag};
  const int threads = 256;
  const int64_t grid = grid_for(num_tokens * num_kv_heads * a.vec_per_row, threads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (vb) {
    case 16: kv_append_kernel<16><<<grid, threads, 0, s>>>(a); break;
    case 8: kv_append_kernel<8><<<grid, threads, 0, s>>>(a); break;
    case 4: kv_append_kernel<4><<<grid, threads, 0, s>>>(a); break;
    default: kv_append_kernel<2><<<grid, threads, 0, s>>>(a); break;
  }
  bump_stat(kStatAppend);
  return cuda_status(cudaGetLastError(), "kv_append launch");
}

extern "C" int pkv_kv_append_positions(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                                       const void* value, int64_t value_stride_token, int64_t value_stride_head,
                                       const int64_t* block_table, int64_t table_len, int64_t start,
                                       int64_t num_tokens, void* key_pool, void* value_pool, int64_t num_pages,
                                       int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                                       int64_t stride_page, int64_t stride_head, int64_t stride_slot, int dtype,
                                       int32_t* error_flag, void* stream) {
  clear_error();
  const int es = dtype_size(dtype);
  PKV_REQUIRE(es > 0, "kv_append_positions: unsupported dtype %d", dtype);
  PKV_REQUIRE(num_tokens >= 0 && start >= 0 && table_len >= 0, "kv_append_positions: negative size");
  PKV_REQUIRE(num_kv_heads > 0 && head_dim > 0 && block_size > 0 && num_pages > 0,
              "kv_append_positions: heads, head_dim, block_size and num_pages must be positive");
  PKV_REQUIRE(start + num_tokens <= table_len * block_size,
              "kv_append_positions: positions [%lld, %lld) exceed the table's %lld blocks",
              static_cast<long long>(start), static_cast<long long>(start + num_tokens),
              static_cast<long long>(table_len));
  if (num_tokens == 0) return PKV_OK;
  PKV_REQUIRE(key && value && block_table && key_pool && value_pool, "kv_append_positions: null pointer argument");
  const int64_t row_bytes = head_dim * es;
  const int vb = vector_bytes({row_bytes, key_stride_token * es, key_stride_head * es, value_stride_token * es,
                               value_stride_head * es, stride_page * es, stride_head * es, stride_slot * es,
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(key)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(value)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(key_pool)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(value_pool))},
                              es);
  AppendArgs a{static_cast<const char*>(key), static_cast<const char*>(value),
               key_stride_token * es, key_stride_head * es, value_stride_token * es, value_stride_head * es,
               nullptr, block_table, table_len, start, num_tokens, static_cast<char*>(key_pool),
               static_cast<char*>(value_pool), num_pages * block_size, block_size, stride_page * es,
               stride_head * es, stride_slot * es, num_kv_heads, row_bytes / vb, error_flag};
  const int threads = 256;
  const int64_t grid = grid_for(num_tokens * num_kv_heads * a.vec_per_row, threads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (vb) {
    case 16: kv_append_kernel<16><<<grid, threads, 0, s>>>(a); break;
    case 8: kv_append_kernel<8><<<grid, threads, 0, s>>>(a); break;
    case 4: kv_append_kernel<4><<<grid, threads, 0, s>>>(a); break;
    default: kv_append_kernel<2><<<grid, threads, 0, s>>>(a); break;
  }
  bump_stat(kStatAppend);
  return cuda_status(cudaGetLastError(), "kv_append_positions launch");
}

extern "C" int pkv_gather_kv(const void* key_pool, const void* value_pool, int64_t num_pages, int64_t num_kv_heads,
                             int64_t block_size, int64_t head_dim, int64_t stride_page, int64_t stride_head,
                             int64_t stride_slot, const void* block_tables, int64_t table_stride,
                             int64_t max_blocks, const void* seq_lens, int index_dtype, int64_t batch,
                             int64_t max_len, void* key_out, void* value_out, int64_t out_stride_batch,
                             int64_t out_stride_head, int64_t out_stride_token, int dtype, int32_t* error_flag,
                             void* stream) {
  clear_error();
  const int es = dtype_size(dtype);
  PKV_REQUIRE(es > 0, "gather_kv: unsupported dtype %d", dtype);
  PKV_REQUIRE(index_dtype == PKV_INDEX_I32 || index_dtype == PKV_INDEX_I64, "gather_kv: bad index dtype");
  PKV_REQUIRE(batch >= 0 && max_len >= 0 && num_kv_heads > 0 && head_dim > 0 && block_size > 0,
              "gather_kv: bad sizes");
  if (batch == 0 || max_len == 0) return PKV_OK;
  PKV_REQUIRE(key_pool && value_pool && block_tables && seq_lens && key_out && value_out,
              "gather_kv: null pointer argument");
  const int64_t row_bytes = head_dim * es;
  const int vb = vector_bytes({row_bytes, stride_page * es, stride_head * es, stride_slot * es,
                               out_stride_batch * es, out_stride_head * es, out_stride_token * es,
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(key_pool)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(value_pool)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(key_out)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(value_out))},
                              es);
  const int threads = 256;
  const int64_t vpr = row_bytes / vb;
  const int64_t grid = grid_for(batch * num_kv_heads * max_len * vpr, threads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto launch = [&](auto idx_tag) {
    using I = decltype(idx_tag);
    GatherArgs<I> a{static_cast<const char*>(key_pool), static_cast<const char*>(value_pool), num_pages, block_size,
                    stride_page * es, stride_head * es, stride_slot * es, static_cast<const I*>(block_tables),
                    table_stride, max_blocks, static_cast<const I*>(seq_lens), batch, num_kv_heads, max_len,
                    static_cast<char*>(key_out), static_cast<char*>(value_out), out_stride_batch * es,
                    out_stride_head * es, out_stride_token * es, vpr, error_flag};
    switch (vb) {
      case 16: kv_gather_kernel<16, I><<<grid, threads, 0, s>>>(a); break;
      case 8: kv_gather_kernel<8, I><<<grid, threads, 0, s>>>(a); break;
      case 4: kv_gather_kernel<4, I><<<grid, threads, 0, s>>>(a); break;
      default: kv_gather_kernel<2, I><<<grid, threads, 0, s>>>(a); break;
    }
  };
  if (index_dtype == PKV_INDEX_I32) launch(int32_t{}); else launch(int64_t{});
  bump_stat(kStatGather);
  return cuda_status(cudaGetLastError(), "gather_kv launch");
}

extern "C" int pkv_copy_pages(void* key_pool, void* value_pool, int64_t num_layers, int64_t layer_stride_bytes,
                              int64_t num_pages, int64_t page_stride_bytes, int64_t chunks_per_page,
                              int64_t chunk_stride_bytes, int64_t chunk_bytes, const int32_t* src_pages,
                              const int32_t* dst_pages, int64_t num_pairs, int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE(num_pairs >= 0 && num_layers > 0 && num_pages > 0 && chunks_per_page > 0 && chunk_bytes > 0,
              "copy_pages: bad sizes");
  if (num_pairs == 0 || (key_pool == nullptr && value_pool == nullptr)) return PKV_OK;
  PKV_REQUIRE(src_pages && dst_pages, "copy_pages: null page list");
  PKV_REQUIRE(chunk_bytes % 2 == 0, "copy_pages: chunk_bytes must be even");
  const int vb = vector_bytes({chunk_bytes, layer_stride_bytes, page_stride_bytes, chunk_stride_bytes,
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(key_pool)),
                               static_cast<int64_t>(reinterpret_cast<uintptr_t>(value_pool))},
                              2);
  CopyArgs a{static_cast<char*>(key_pool), static_cast<char*>(value_pool), num_layers, layer_stride_bytes, num_pages,
             page_stride_bytes, chunks_per_page, chunk_stride_bytes, chunk_bytes / vb, src_pages, dst_pages,
             num_pairs, error_flag};
  const int threads = 256;
  const int64_t grid = grid_for(num_layers * num_pairs * chunks_per_page * a.vec_per_chunk / 4 + 1, threads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (vb) {
    case 16: copy_pages_kernel<16><<<grid, threads, 0, s>>>(a); break;
    case 8: copy_pages_kernel<8><<<grid, threads, 0, s>>>(a); break;
    case 4: copy_pages_kernel<4><<<grid, threads, 0, s>>>(a); break;
    default: copy_pages_kernel<2><<<grid, threads, 0, s>>>(a); break;
  }
  bump_stat(kStatCopyPages);
  return cuda_status(cudaGetLastError(), "copy_pages launch");
}

extern "C" int pkv_decode_slot_mapping_layers(const void* block_tables, int64_t table_stride, int64_t max_blocks,
                                              void* seq_lens, int index_dtype, int64_t batch, int64_t block_size,
                                              int64_t num_pages, int64_t num_layers, int64_t* slot_mapping,
                                              int advance, int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE(index_dtype == PKV_INDEX_I32 || index_dtype == PKV_INDEX_I64, "decode_slot_mapping: bad index dtype");
  PKV_REQUIRE(batch >= 0 && max_blocks > 0 && block_size > 0 && num_pages > 0, "decode_slot_mapping: bad sizes");
  PKV_REQUIRE(num_layers >= 1, "decode_slot_mapping: num_layers must be positive");
  if (batch == 0) return PKV_OK;
  PKV_REQUIRE(block_tables && seq_lens && slot_mapping, "decode_slot_mapping: null pointer argument");
  const int threads = 256;
  const int64_t grid = ceil_div(batch, threads);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (index_dtype == PKV_INDEX_I32) {
    decode_slots_kernel<int32_t><<<grid, threads, 0, s>>>(static_cast<const int32_t*>(block_tables), table_stride,
                                                          max_blocks, static_cast<int32_t*>(seq_lens), batch,
                                                          block_size, num_pages, slot_mapping, advance, num_layers,
                                                          error_flag);
  } else {
    decode_slots_kernel<int64_t><<<grid, threads, 0, s>>>(static_cast<const int64_t*>(block_tables), table_stride,
                                                          max_blocks, static_cast<int64_t*>(seq_lens), batch,
                                                          block_size, num_pages, slot_mapping, advance, num_layers,
                                                          error_flag);
  }
  bump_stat(kStatAppend);
  return cuda_status(cudaGetLastError(), "decode_slot_mapping launch");
}

extern "C" int pkv_decode_slot_mapping(const void* block_tables, int64_t table_stride, int64_t max_blocks,
                                       void* seq_lens, int index_dtype, int64_t batch, int64_t block_size,
                                       int64_t num_pages, int64_t* slot_mapping, int advance, int32_t* error_flag,
                                       void* stream) {
  return pkv_decode_slot_mapping_layers(block_tables, table_stride, max_blocks, seq_lens, index_dtype, batch,
                                        block_size, num_pages, 1, slot_mapping, advance, error_flag, stream);
}

extern "C" int pkv_kv_append_fp8(const void* key, int64_t key_stride_token, int64_t key_stride_head,
                                 const void* value, int64_t value_stride_token, int64_t value_stride_head,
                                 const int64_t* slot_mapping, int64_t num_tokens, void* key_pool, void* value_pool,
                                 float* key_scales, float* value_scales, int64_t scale_stride_page,
                                 int64_t scale_stride_head, int64_t num_pages, int64_t num_kv_heads,
                                 int64_t block_size, int64_t head_dim, int64_t stride_page, int64_t stride_head,
                                 int64_t stride_slot, int dtype, int32_t* error_flag, void* stream) {
  clear_error();
  const int es = dtype_size(dtype);
  PKV_REQUIRE(es > 0, "kv_append_fp8: unsupported dtype %d", dtype);
  PKV_REQUIRE(num_tokens >= 0, "kv_append_fp8: num_tokens must be non-negative");
  PKV_REQUIRE(num_kv_heads > 0 && block_size > 0 && num_pages > 0,
              "kv_append_fp8: heads, block_size and num_pages must be positive");
  PKV_REQUIRE(head_dim == 64 || head_dim == 128 || head_dim == 256 || head_dim == 512 || head_dim == 1024,
              "kv_append_fp8: head_dim must be 64, 128, 256, 512 or 1024");
  if (num_tokens == 0) return PKV_OK;
  PKV_REQUIRE(key && value && slot_mapping && key_pool && value_pool && key_scales && value_scales,
              "kv_append_fp8: null pointer argument");
  const int64_t epl = head_dim / 32;
  PKV_REQUIRE((reinterpret_cast<uintptr_t>(key_pool) | reinterpret_cast<uintptr_t>(value_pool)) % 4 == 0 &&
                  stride_page % 4 == 0 && stride_head % 4 == 0 && stride_slot % 4 == 0,
              "kv_append_fp8: fp8 pools need 4-byte aligned rows");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  bump_stat(kStatAppendFp8);
  auto run = [&](auto tag, auto epl_tag) -> int {
    using T = decltype(tag);
    constexpr int EPL = decltype(epl_tag)::value;
    Fp8AppendArgs<T, EPL> a{static_cast<const T*>(key), static_cast<const T*>(value), key_stride_token,
                            key_stride_head, value_stride_token, value_stride_head, slot_mapping, num_tokens,
                            static_cast<uint8_t*>(key_pool), static_cast<uint8_t*>(value_pool), key_scales,
                            value_scales, num_pages * block_size, block_size, stride_page, stride_head,
                            stride_slot, scale_stride_page, scale_stride_head, static_cast<int32_t>(num_kv_heads),
                            error_flag};
    return launch_append_fp8<T, EPL>(a, s);
  };
  auto by_epl = [&](auto tag) -> int {
    switch (epl) {
      case 2: return run(tag, std::integral_constant<int, 2>{});
      case 4: return run(tag, std::integral_constant<int, 4>{});
      case 8: return run(tag, std::integral_constant<int, 8>{});
      case 16: return run(tag, std::integral_constant<int, 16>{});
      default: return run(tag, std::integral_constant<int, 32>{});
    }
  };
  if (dtype == PKV_DTYPE_F32) return by_epl(float{});
  if (dtype == PKV_DTYPE_F16) return by_epl(__half{});
  return by_epl(__nv_bfloat16{});
}
