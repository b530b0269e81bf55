// Chunked-prefill paged causal attention.
//
// Request b appends a chunk of q_b = cu_q[b+1] - cu_q[b] tokens (already written to its pages) at
// absolute positions L_b - q_b .. L_b - 1, where L_b = seq_lens[b] includes the chunk. Query token i
// attends keys [0, L_b - q_b + i] of its pages -- the causal mask of the reference's dense prefill
// (key_pos > query_pos masked, src/tp_runtime.py:716-721) over the prefix pages and the chunk's own.
//
// Tensor-core path (fp16/bf16, head_dim 64/128/256, 8 query heads per KV head, block_size % 16 == 0,
// native-compatible layouts). One CTA owns 16 chunk tokens x the 8 query heads that share one KV head
// (128 GQA-packed rows, so every K/V tile is loaded once for all 8 heads) and streams 32-key tiles
// through a ring of shared-memory stages filled by TMA (the decode kernel's 3-D page-tile boxes).
// Eight warps own 16 rows each (2 tokens x 8 heads): S = Q K^T and O += P V with mma.m16n8k16 (fp32
// accumulators in registers), online softmax per row, causal mask by absolute position. Q (64 KB at
// head_dim 256) stays in shared memory (4-D TMA, 128-byte swizzle). Each warp releases a stage on an
// "empty" mbarrier; lane 0 of warp 0 refills it once all eight have (no separate producer warp, so
// every thread keeps the 255-register budget the 128 output accumulators need).
// bf16 carries P as hi + lo parts (two P.V products), as in decode, so P stays fp32-accurate.
//
// Generic path (every other shape, fp32): CUDA cores, one warp per (query token, query head), online
// softmax over the token's causal key range.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <mutex>

#include "pkv_common.cuh"

namespace pkv {
namespace {

constexpr uint64_t kPrefillWaitNs = 2000000000ull;
constexpr int kPfConsumers = 8;                // warps, 16 rows each
constexpr int kPfThreads = kPfConsumers * 32;
constexpr int kPfTokens = 16;                  // chunk tokens per CTA
constexpr int kPfGroup = 8;                    // query heads per KV head on this path
constexpr int kPfKeys = 32;                    // keys per stage (two 16-row page tiles)

template <int D>
struct PfConfig {
  static constexpr int kTileBytes = 16 * D * 2;             // one 16-key K (or V) page tile
  static constexpr int kStageBytes = 4 * kTileBytes;        // K and V for 32 keys
  static constexpr int kQBytes = kPfTokens * kPfGroup * D * 2;
  static constexpr int kStages = D == 256 ? 3 : 4;
  static constexpr int kSmemBytes = kQBytes + kStages * kStageBytes + 2 * kStages * 8 + 8 + 1024;
};

template <typename I>
struct PfArgs {
  const int32_t* cu_q;
  const I* tables;
  int64_t table_stride;
  int32_t max_blocks;
  const I* seq_lens;
  int32_t batch, num_pages, block_size;
  int32_t rows_per_page, rows_per_head;
  int32_t num_kv_heads;
  float scale_log2;
  void* out;
  int64_t o_st, o_sh;  // elements
  int32_t* error_flag;
};

template <typename T, typename I, int D>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const PfArgs<I> a) {
  using Cfg = PfConfig<D>;
  constexpr int NST = Cfg::kStages;
  constexpr int NB = D / 64;
  constexpr int ND = D / 8;  // n-tiles of the output
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* qs = smem;
  uint8_t* stages = smem + Cfg::kQBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(stages + NST * Cfg::kStageBytes);
  uint64_t* empty = full + NST;
  uint64_t* qbar = empty + NST;

  const int b = blockIdx.z, kvh = blockIdx.y;
  const int q_begin = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - q_begin;
  const int t0 = blockIdx.x * kPfTokens;
  if (t0 >= q_len) return;
  int64_t len = load_index(a.seq_lens, b);
  const int64_t cap = static_cast<int64_t>(a.max_blocks) * a.block_size;
  if (len > cap) len = cap;
  const int64_t pos0 = len - q_len;  // absolute position of chunk token 0
  const int ntok = min(kPfTokens, q_len - t0);
  const int64_t last_pos = pos0 + t0 + ntok - 1;
  const int n_tiles = last_pos < 0 ? 0 : static_cast<int>((last_pos + kPfKeys) / kPfKeys);  // 32-key tiles
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&qmap);
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kPfConsumers);
    }
    mbar_init(qbar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---------------- loads (lane 0 of warp 0)
  const I* trow = a.tables + static_cast<int64_t>(b) * a.table_stride;
  const int tiles_per_page = a.block_size >> 4;
  const int64_t pages = (len + a.block_size - 1) / a.block_size;
  const uint64_t policy = policy_evict_first();
  bool bad_page = false;
  // Issues the K/V page tiles of stage tile j (keys 32j .. 32j + 31) into stage j % NST.
  auto issue = [&](int j) {
    const int s = j % NST;
    uint8_t* st = stages + s * Cfg::kStageBytes;
    int64_t page_of[2];
    int issued = 0;
    for (int h = 0; h < 2; ++h) {
      const int tile = 2 * j + h;  // 16-key page tile index
      const int page_local = tile / tiles_per_page;
      page_of[h] = -1;
      if (page_local >= pages) continue;  // beyond the context: the consumers mask these keys
      const int64_t page = load_index(trow, page_local);
      if (page < 0 || page >= a.num_pages) {
        bad_page = true;
        continue;
      }
      page_of[h] = page;
      ++issued;
    }
    mbar_arrive_expect_tx(&full[s], issued * 2 * Cfg::kTileBytes);
    for (int h = 0; h < 2; ++h) {
      if (page_of[h] < 0) continue;
      const int tile = 2 * j + h;
      const int page_local = tile / tiles_per_page;
      const int row = static_cast<int>(page_of[h]) * a.rows_per_page + kvh * a.rows_per_head +
                      (tile - page_local * tiles_per_page) * 16;
      tma_load_3d(st + h * Cfg::kTileBytes, &kmap, &full[s], 0, row, 0, policy);
      tma_load_3d(st + (2 + h) * Cfg::kTileBytes, &vmap, &full[s], 0, row, 0, policy);
    }
  };
  if (threadIdx.x == 0) {
    mbar_arrive_expect_tx(qbar, Cfg::kQBytes);
    tma_load_4d(qs, &qmap, qbar, 0, kvh * kPfGroup, q_begin + t0, 0, policy_evict_last());
    for (int j = 0; j < NST && j < n_tiles; ++j) issue(j);
  }

  // ---------------- warps: rows 16*warp .. +16 = tokens 2*warp, 2*warp+1 x 8 heads
  const int g = lane >> 2, t = lane & 3;
  const int tok_lo = 2 * warp, tok_hi = 2 * warp + 1;  // chunk-tile tokens of rows g and g+8
  const int64_t qpos_lo = pos0 + t0 + tok_lo, qpos_hi = pos0 + t0 + tok_hi;
  const uint32_t qbase = smem_u32(qs);
  if (!mbar_wait_bounded(qbar, 0, kPrefillWaitNs)) {
    if (lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
    return;
  }
  float m_lo = kNegInf, m_hi = kNegInf, l_lo = 0.f, l_hi = 0.f;
  float o[ND][4];
#pragma unroll
  for (int n = 0; n < ND; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  const int row_base = 16 * warp;
  // ldmatrix lane roles
  const int lrow = lane & 7, lsel = lane >> 3;

  for (int j = 0; j < n_tiles; ++j) {
    const int s = j % NST;
    if (warp == 0 && j >= 1 && j - 1 + NST < n_tiles) {
      // refill the stage tile j - 1 used, once every warp has released it
      bool freed = true;
      if (lane == 0) {
        freed = mbar_wait_bounded(&empty[(j - 1) % NST], ((j - 1) / NST) & 1, kPrefillWaitNs);
        if (freed) issue(j - 1 + NST);
      }
      if (!__shfl_sync(0xffffffffu, freed, 0)) {
        if (lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
        return;
      }
    }
    const bool landed = mbar_wait_bounded(&full[s], (j / NST) & 1, kPrefillWaitNs);
    if (!__all_sync(0xffffffffu, landed)) {
      if (lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
      return;
    }
    const uint32_t kb = smem_u32(stages + s * Cfg::kStageBytes);
    const uint32_t vb = kb + 2 * Cfg::kTileBytes;
    // ---- S = Q K^T : 16 rows x 32 keys (4 n-tiles)
    float sacc[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) sacc[n][0] = sacc[n][1] = sacc[n][2] = sacc[n][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < D / 16; ++ks) {
      const int chunk = 2 * ks;  // 8-element chunk of d for this k-step
      // Q: matrices (rows 0-7, chunk), (rows 8-15, chunk), (rows 0-7, chunk+1), (rows 8-15, chunk+1)
      uint32_t qa0, qa1, qa2, qa3;
      {
        const int r = row_base + lrow + ((lsel & 1) << 3);
        const int c = chunk + (lsel >> 1);
        ldsm_x4(qbase + (c >> 3) * (kPfTokens * kPfGroup * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4), qa0, qa1,
                qa2, qa3);
      }
#pragma unroll
      for (int np = 0; np < 2; ++np) {  // pairs of 8-key n-tiles = one 16-key page tile
        // K: matrices (keys 0-7, chunk), (keys 0-7, chunk+1), (keys 8-15, chunk), (keys 8-15, chunk+1)
        const int key = lrow + ((lsel >> 1) << 3);
        const int c = chunk + (lsel & 1);
        uint32_t k0, k1, k2, k3;
        ldsm_x4(kb + np * Cfg::kTileBytes + (c >> 3) * 2048 + key * 128 + (((c & 7) ^ (key & 7)) << 4), k0, k1,
                k2, k3);
        mma_16816<T>(sacc[2 * np], qa0, qa1, qa2, qa3, k0, k1);
        mma_16816<T>(sacc[2 * np + 1], qa0, qa1, qa2, qa3, k2, k3);
      }
    }
    // ---- causal mask, online softmax (rows g: token tok_lo, g+8: token tok_hi)
    const int64_t key0 = static_cast<int64_t>(j) * kPfKeys;
    float mx_lo = kNegInf, mx_hi = kNegInf;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t kp = key0 + 8 * n + 2 * t + e;
        float vlo = sacc[n][e] * a.scale_log2, vhi = sacc[n][2 + e] * a.scale_log2;
        if (kp > qpos_lo || kp >= len) vlo = kNegInf;
        if (kp > qpos_hi || kp >= len) vhi = kNegInf;
        sacc[n][e] = vlo;
        sacc[n][2 + e] = vhi;
        mx_lo = fmaxf(mx_lo, vlo);
        mx_hi = fmaxf(mx_hi, vhi);
      }
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
      mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, off));
      mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, off));
    }
    const float mn_lo = fmaxf(m_lo, mx_lo), mn_hi = fmaxf(m_hi, mx_hi);
    const float base_lo = mn_lo == kNegInf ? 0.f : mn_lo, base_hi = mn_hi == kNegInf ? 0.f : mn_hi;
    const float alpha_lo = fast_exp2(m_lo - base_lo), alpha_hi = fast_exp2(m_hi - base_hi);
    m_lo = mn_lo;
    m_hi = mn_hi;
    float ps_lo = 0.f, ps_hi = 0.f;
#pragma unroll
    for (int n = 0; n < 4; ++n) {
      sacc[n][0] = fast_exp2(sacc[n][0] - base_lo);
      sacc[n][1] = fast_exp2(sacc[n][1] - base_lo);
      sacc[n][2] = fast_exp2(sacc[n][2] - base_hi);
      sacc[n][3] = fast_exp2(sacc[n][3] - base_hi);
      ps_lo += sacc[n][0] + sacc[n][1];
      ps_hi += sacc[n][2] + sacc[n][3];
    }
    l_lo = l_lo * alpha_lo + ps_lo;
    l_hi = l_hi * alpha_hi + ps_hi;
    if (__any_sync(0xffffffffu, alpha_lo != 1.f || alpha_hi != 1.f)) {
#pragma unroll
      for (int n = 0; n < ND; ++n) {
        o[n][0] *= alpha_lo; o[n][1] *= alpha_lo; o[n][2] *= alpha_hi; o[n][3] *= alpha_hi;
      }
    }
    // ---- O += P V : two 16-key k-steps (one per page tile). Keys at or past the context end have
    // P = 0, but their V rows were never written (or not loaded at all), and 0 * NaN is NaN: whole
    // tiles past the end are skipped and partial ones have those V rows zeroed.
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const int64_t kt0 = key0 + 16 * kk;
      if (kt0 >= len) continue;
      uint32_t mlo = 0xffffffffu, mhi = 0xffffffffu;
      if (kt0 + 16 > len) {
        mlo = (kt0 + 2 * t < len ? 0x0000ffffu : 0u) | (kt0 + 2 * t + 1 < len ? 0xffff0000u : 0u);
        mhi = (kt0 + 2 * t + 8 < len ? 0x0000ffffu : 0u) | (kt0 + 2 * t + 9 < len ? 0xffff0000u : 0u);
      }
      const uint32_t a0 = pack2<T>(sacc[2 * kk][0], sacc[2 * kk][1]);
      const uint32_t a1 = pack2<T>(sacc[2 * kk][2], sacc[2 * kk][3]);
      const uint32_t a2 = pack2<T>(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1]);
      const uint32_t a3 = pack2<T>(sacc[2 * kk + 1][2], sacc[2 * kk + 1][3]);
      uint32_t l0 = 0, l1 = 0, l2 = 0, l3 = 0;
      if constexpr (kSplitP<T>) {
        const float2 h0 = unpack2<T>(a0), h1 = unpack2<T>(a1), h2 = unpack2<T>(a2), h3 = unpack2<T>(a3);
        l0 = pack2<T>(sacc[2 * kk][0] - h0.x, sacc[2 * kk][1] - h0.y);
        l1 = pack2<T>(sacc[2 * kk][2] - h1.x, sacc[2 * kk][3] - h1.y);
        l2 = pack2<T>(sacc[2 * kk + 1][0] - h2.x, sacc[2 * kk + 1][1] - h2.y);
        l3 = pack2<T>(sacc[2 * kk + 1][2] - h3.x, sacc[2 * kk + 1][3] - h3.y);
      }
      const uint32_t vt = vb + kk * Cfg::kTileBytes;
#pragma unroll
      for (int np = 0; np < ND / 2; ++np) {  // pairs of 8-column n-tiles
        // V^T fragments via ldmatrix.trans: (keys 0-7, chunk 2np), (keys 8-15, chunk 2np),
        // (keys 0-7, chunk 2np+1), (keys 8-15, chunk 2np+1)
        const int key = lrow + ((lsel & 1) << 3);
        const int c = 2 * np + (lsel >> 1);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_trans(vt + (c >> 3) * 2048 + key * 128 + (((c & 7) ^ (key & 7)) << 4), v0, v1, v2, v3);
        v0 &= mlo; v1 &= mhi; v2 &= mlo; v3 &= mhi;
        mma_16816<T>(o[2 * np], a0, a1, a2, a3, v0, v1);
        mma_16816<T>(o[2 * np + 1], a0, a1, a2, a3, v2, v3);
        if constexpr (kSplitP<T>) {
          mma_16816<T>(o[2 * np], l0, l1, l2, l3, v0, v1);
          mma_16816<T>(o[2 * np + 1], l0, l1, l2, l3, v2, v3);
        }
      }
    }
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  if (threadIdx.x == 0 && bad_page) raise_device_error(a.error_flag, PKV_DEVERR_PAGE_OUT_OF_RANGE);
  // ---- epilogue: normalise and store rows of valid tokens
#pragma unroll
  for (int off = 1; off < 4; off <<= 1) {
    l_lo += __shfl_xor_sync(0xffffffffu, l_lo, off);
    l_hi += __shfl_xor_sync(0xffffffffu, l_hi, off);
  }
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f, inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
  T* obase = static_cast<T*>(a.out);
  const int head = kvh * kPfGroup + g;
  if (tok_lo < ntok) {
    T* orow = obase + static_cast<int64_t>(q_begin + t0 + tok_lo) * a.o_st + head * a.o_sh;
#pragma unroll
    for (int n = 0; n < ND; ++n)
      *reinterpret_cast<uint32_t*>(orow + 8 * n + 2 * t) = pack2<T>(o[n][0] * inv_lo, o[n][1] * inv_lo);
  }
  if (tok_hi < ntok) {
    T* orow = obase + static_cast<int64_t>(q_begin + t0 + tok_hi) * a.o_st + head * a.o_sh;
#pragma unroll
    for (int n = 0; n < ND; ++n)
      *reinterpret_cast<uint32_t*>(orow + 8 * n + 2 * t) = pack2<T>(o[n][2] * inv_hi, o[n][3] * inv_hi);
  }
}

// ---- generic path ----------------------------------------------------------------------------------------
template <typename I>
struct PfGenArgs {
  const void* q;
  int64_t q_st, q_sh;
  const int32_t* cu_q;
  int32_t batch;
  int64_t total_q;
  const void* kpool;
  const void* vpool;
  int64_t num_pages, block_size, head_dim, sp, sh, ss;
  const I* tables;
  int64_t table_stride, max_blocks;
  const I* seq_lens;
  int32_t num_q_heads, group;
  float scale_log2;
  void* out;
  int64_t o_st, o_sh;
  int32_t* error_flag;
};

// One warp per (query token, query head): online softmax over the token's causal key range.
template <typename T, typename I, int MAXK>
__global__ void __launch_bounds__(128) prefill_generic_kernel(const PfGenArgs<I> a) {
  const int64_t item = (static_cast<int64_t>(blockIdx.x) * 4 + (threadIdx.x >> 5));
  const int lane = threadIdx.x & 31;
  if (item >= a.total_q * a.num_q_heads) return;
  const int64_t qi = item / a.num_q_heads;
  const int h = static_cast<int>(item - qi * a.num_q_heads);
  int b = 0;
  while (b + 1 < a.batch && a.cu_q[b + 1] <= qi) ++b;
  const int q_len = a.cu_q[b + 1] - a.cu_q[b];
  int64_t len = load_index(a.seq_lens, b);
  const int64_t cap = a.max_blocks * a.block_size;
  if (len > cap) len = cap;
  const int64_t qpos = len - q_len + (qi - a.cu_q[b]);
  const int D = static_cast<int>(a.head_dim);
  const int kvh = h / a.group;
  const T* qrow = static_cast<const T*>(a.q) + qi * a.q_st + h * a.q_sh;
  float q[MAXK], acc[MAXK];
#pragma unroll
  for (int k = 0; k < MAXK; ++k) {
    const int d = 32 * k + lane;
    q[k] = d < D ? Elem<T>::to_f(qrow[d]) : 0.f;
    acc[k] = 0.f;
  }
  float m = kNegInf, l = 0.f;
  const I* trow = a.tables + static_cast<int64_t>(b) * a.table_stride;
  const int es = sizeof(T);
  for (int64_t kp = 0; kp <= qpos && kp < len; ++kp) {
    const int64_t logical = kp / a.block_size;
    const int64_t page = load_index(trow, logical);
    if (page < 0 || page >= a.num_pages) {
      if (lane == 0) raise_device_error(a.error_flag, PKV_DEVERR_PAGE_OUT_OF_RANGE);
      continue;
    }
    const int64_t off = (page * a.sp + kvh * a.sh + (kp - logical * a.block_size) * a.ss) * es;
    const T* krow = reinterpret_cast<const T*>(static_cast<const char*>(a.kpool) + off);
    const T* vrow = reinterpret_cast<const T*>(static_cast<const char*>(a.vpool) + off);
    float part = 0.f;
#pragma unroll
    for (int k = 0; k < MAXK; ++k) {
      const int d = 32 * k + lane;
      if (d < D) part = fmaf(q[k], Elem<T>::to_f(krow[d]), part);
    }
#pragma unroll
    for (int off2 = 16; off2 > 0; off2 >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off2);
    const float sc = part * a.scale_log2;
    const float mn = fmaxf(m, sc);
    const float base = mn == kNegInf ? 0.f : mn;
    const float alpha = fast_exp2(m - base), p = fast_exp2(sc - base);
    l = l * alpha + p;
    m = mn;
#pragma unroll
    for (int k = 0; k < MAXK; ++k) {
      const int d = 32 * k + lane;
      acc[k] = fmaf(p, d < D ? Elem<T>::to_f(vrow[d]) : 0.f, acc[k] * alpha);
    }
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  T* orow = static_cast<T*>(a.out) + qi * a.o_st + h * a.o_sh;
#pragma unroll
  for (int k = 0; k < MAXK; ++k) {
    const int d = 32 * k + lane;
    if (d < D) orow[d] = Elem<T>::from_f(acc[k] * inv);
  }
}

// ---- host ------------------------------------------------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 encoder() {
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

int encode(CUtensorMap* map, const void* base, int dtype, int rank, const cuuint64_t* dims, const cuuint64_t* strides,
           const cuuint32_t* box) {
  auto fn = encoder();
  if (fn == nullptr) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return PKV_ERR_CUDA;
  }
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = fn(map, dtype == PKV_DTYPE_F16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                  rank, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult %d", static_cast<int>(r));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

template <typename T, typename I, int D>
int launch_prefill_tc(const CUtensorMap& qm, const CUtensorMap& km, const CUtensorMap& vm, const PfArgs<I>& a,
                      int64_t max_q_len, cudaStream_t s) {
  using Cfg = PfConfig<D>;
  auto kern = prefill_tc_kernel<T, I, D>;
  static bool configured = false;
  if (!configured) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes);
    if (e != cudaSuccess) return cuda_status(e, "prefill_tc_kernel smem attribute");
    configured = true;
  }
  const dim3 grid(static_cast<unsigned>((max_q_len + kPfTokens - 1) / kPfTokens), a.num_kv_heads, a.batch);
  kern<<<grid, kPfThreads, Cfg::kSmemBytes, s>>>(qm, km, vm, a);
  return cuda_status(cudaGetLastError(), "prefill_tc_kernel launch");
}

template <typename I>
int run_prefill(const void* query, int64_t q_st, int64_t q_sh, const int32_t* cu_q, int64_t total_q,
                int64_t max_q_len, const void* kpool, const void* vpool, int64_t num_pages, int64_t num_kv_heads,
                int64_t block_size, int64_t head_dim, int64_t sp, int64_t sh, int64_t ss, const void* tables,
                int64_t table_stride, int64_t max_blocks, const void* seq_lens, int64_t batch, int64_t num_q_heads,
                float scale, void* out, int64_t o_st, int64_t o_sh, int dtype, int32_t* error_flag,
                cudaStream_t stream) {
  const int64_t group = num_q_heads / num_kv_heads;
  const float scale_log2 = scale * kLog2e;
  const uintptr_t align = reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(kpool) |
                          reinterpret_cast<uintptr_t>(vpool) | reinterpret_cast<uintptr_t>(out);
  const int64_t rows = (num_pages - 1) * (sp / head_dim) + (num_kv_heads - 1) * (sh / head_dim) + block_size;
  const bool tc_ok = (dtype == PKV_DTYPE_F16 || dtype == PKV_DTYPE_BF16) &&
                     (head_dim == 64 || head_dim == 128 || head_dim == 256) && group == kPfGroup &&
                     block_size % 16 == 0 && ss == head_dim && sp % head_dim == 0 && sh % head_dim == 0 &&
                     q_sh == head_dim && q_st % 8 == 0 && o_st % 2 == 0 && o_sh % 2 == 0 && align % 16 == 0 &&
                     rows < (1ll << 31) && total_q < (1ll << 31) && batch < 65536 && num_kv_heads < 65536;
  bump_stat(kStatPrefill);
  if (tc_ok) {
    CUtensorMap qm, km, vm;
    const cuuint64_t qdims[4] = {64, static_cast<cuuint64_t>(num_q_heads), static_cast<cuuint64_t>(total_q),
                                 static_cast<cuuint64_t>(head_dim / 64)};
    const cuuint64_t qstr[3] = {static_cast<cuuint64_t>(head_dim * 2), static_cast<cuuint64_t>(q_st * 2), 128};
    const cuuint32_t qbox[4] = {64, kPfGroup, kPfTokens, static_cast<cuuint32_t>(head_dim / 64)};
    int st = encode(&qm, query, dtype, 4, qdims, qstr, qbox);
    if (st != PKV_OK) return st;
    const cuuint64_t kdims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(head_dim / 64)};
    const cuuint64_t kstr[2] = {static_cast<cuuint64_t>(head_dim * 2), 128};
    const cuuint32_t kbox[3] = {64, 16, static_cast<cuuint32_t>(head_dim / 64)};
    st = encode(&km, kpool, dtype, 3, kdims, kstr, kbox);
    if (st != PKV_OK) return st;
    st = encode(&vm, vpool, dtype, 3, kdims, kstr, kbox);
    if (st != PKV_OK) return st;
    PfArgs<I> a{cu_q, static_cast<const I*>(tables), table_stride, static_cast<int32_t>(max_blocks),
                static_cast<const I*>(seq_lens), static_cast<int32_t>(batch), static_cast<int32_t>(num_pages),
                static_cast<int32_t>(block_size), static_cast<int32_t>(sp / head_dim),
                static_cast<int32_t>(sh / head_dim), static_cast<int32_t>(num_kv_heads), scale_log2, out, o_st, o_sh,
                error_flag};
    if (dtype == PKV_DTYPE_F16) {
      if (head_dim == 64) return launch_prefill_tc<__half, I, 64>(qm, km, vm, a, max_q_len, stream);
      if (head_dim == 128) return launch_prefill_tc<__half, I, 128>(qm, km, vm, a, max_q_len, stream);
      return launch_prefill_tc<__half, I, 256>(qm, km, vm, a, max_q_len, stream);
    }
    if (head_dim == 64) return launch_prefill_tc<__nv_bfloat16, I, 64>(qm, km, vm, a, max_q_len, stream);
    if (head_dim == 128) return launch_prefill_tc<__nv_bfloat16, I, 128>(qm, km, vm, a, max_q_len, stream);
    return launch_prefill_tc<__nv_bfloat16, I, 256>(qm, km, vm, a, max_q_len, stream);
  }
  PfGenArgs<I> g{query, q_st, q_sh, cu_q, static_cast<int32_t>(batch), total_q, kpool, vpool, num_pages, block_size,
                 head_dim, sp, sh, ss, static_cast<const I*>(tables), table_stride, max_blocks,
                 static_cast<const I*>(seq_lens), static_cast<int32_t>(num_q_heads), static_cast<int32_t>(group),
                 scale_log2, out, o_st, o_sh, error_flag};
  const int64_t grid = (total_q * num_q_heads + 3) / 4;
  auto launch = [&](auto tag) {
    using T = decltype(tag);
    if (head_dim <= 256)
      prefill_generic_kernel<T, I, 8><<<grid, 128, 0, stream>>>(g);
    else
      prefill_generic_kernel<T, I, 32><<<grid, 128, 0, stream>>>(g);
  };
  if (dtype == PKV_DTYPE_F32) launch(float{});
  else if (dtype == PKV_DTYPE_F16) launch(__half{});
  else launch(__nv_bfloat16{});
  return cuda_status(cudaGetLastError(), "prefill_generic_kernel launch");
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int pkv_paged_prefill(const void* query, int64_t q_stride_token, int64_t q_stride_head, const int32_t* cu_q,
                                 int64_t total_q, int64_t max_q_len, const void* key_pool, const void* value_pool,
                                 int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                                 int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                                 const void* block_tables, int64_t table_stride, int64_t max_blocks,
                                 const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                                 float scale, void* output, int64_t o_stride_token, int64_t o_stride_head, int dtype,
                                 int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE(dtype_size(dtype) > 0, "paged_prefill: unsupported dtype %d", dtype);
  PKV_REQUIRE(index_dtype == PKV_INDEX_I32 || index_dtype == PKV_INDEX_I64, "paged_prefill: bad index dtype");
  PKV_REQUIRE(batch >= 0 && total_q >= 0 && max_q_len >= 0, "paged_prefill: bad sizes");
  PKV_REQUIRE(num_kv_heads > 0 && num_q_heads > 0 && num_q_heads % num_kv_heads == 0,
              "paged_prefill: num_q_heads must be a positive multiple of num_kv_heads");
  PKV_REQUIRE(head_dim > 0 && head_dim <= 1024 && block_size > 0 && num_pages > 0 && max_blocks > 0,
              "paged_prefill: head_dim, block_size, num_pages and max_blocks must be positive");
  PKV_REQUIRE(std::isfinite(scale), "paged_prefill: scale must be finite");
  if (batch == 0 || total_q == 0) return PKV_OK;
  PKV_REQUIRE(query && cu_q && key_pool && value_pool && block_tables && seq_lens && output,
              "paged_prefill: null pointer argument");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (index_dtype == PKV_INDEX_I32)
    return run_prefill<int32_t>(query, q_stride_token, q_stride_head, cu_q, total_q, max_q_len, key_pool, value_pool,
                                num_pages, num_kv_heads, block_size, head_dim, stride_page, stride_head, stride_slot,
                                block_tables, table_stride, max_blocks, seq_lens, batch, num_q_heads, scale, output,
                                o_stride_token, o_stride_head, dtype, error_flag, s);
  return run_prefill<int64_t>(query, q_stride_token, q_stride_head, cu_q, total_q, max_q_len, key_pool, value_pool,
                              num_pages, num_kv_heads, block_size, head_dim, stride_page, stride_head, stride_slot,
                              block_tables, table_stride, max_blocks, seq_lens, batch, num_q_heads, scale, output,
                              o_stride_token, o_stride_head, dtype, error_flag, s);
}
