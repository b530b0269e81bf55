// Chunked-prefill paged causal attention.
//
// Request b appends a chunk of q_b = cu_q[b+1] - cu_q[b] tokens (already written to its pages) at
// absolute positions L_b - q_b .. L_b - 1, where L_b = seq_lens[b] includes the chunk. Query token i
// attends keys [0, L_b - q_b + i] of its pages -- the causal mask of the reference's dense prefill
// (key_pos > query_pos masked, src/tp_runtime.py:716-721) over the prefix pages and the chunk's own.
//
// Tensor-core path (fp16/bf16, head_dim 64/128/256, G = Hq/Hkv in {1, 2, 4, 8, 16}, block_size % 16 == 0,
// native-compatible pool layout, scale > 0): tcgen05 MMAs with operands and accumulators in tensor memory.
// One CTA owns 128 GQA-packed rows -- 128/G chunk tokens x the G query heads that share one KV head, row =
// token * G + head -- so every K/V byte is loaded once for all G heads. Tensor memory (512 columns) holds
//   O     [0, D)                fp32 accumulator, 128 lanes (rows) x head_dim
//   Q     [D, 1.5 D)            the rows' queries, two 16-bit values per column (A operand of S = Q K^T)
//   S/P   2 x 64 columns        fp32 scores of a 64-key tile; the softmax overwrites them in place with
//                               P (16-bit, hi part in the first 32 columns, lo part in the last 32)
// so shared memory holds only K and V: 64-key tiles in separate rings filled by TMA from the page table
// (K as 2-D 16-row boxes per 64-column chunk, one K-major operand of 64 rows per tile; V as the decode
// kernel's 3-D page-tile boxes, an MN-major operand).
// Roles (384 threads):
//   warp 0        K loads (lanes 0-3, one 16-key page tile each);
//   warp 2        V loads (same page tiles);
//   warp 1        allocates tensor memory; lane 0 issues S_j = Q K_j^T into S/P buffer j % 2 once K_j has
//                 landed and PV_{j-2} (the last reader of that buffer) has completed;
//   warp 11       lane 0 issues O += P_j V_j (A operand P_j in tensor memory) once the softmax has written
//                 P_j. Two issuers keep the tensor pipe fed: the hardware accepts only a few MMAs ahead of
//                 execution, and each issuer's commits and barrier waits overlap the other's MMAs. The
//                 softmax of tile j+1 overlaps PV_j;
//   warps 3-10    two threads per row (tensor-memory lane = row; warps w and w + 4 share lanes and split
//                 a tile's 64 keys). They first copy the rows' queries from global memory into tensor
//                 memory. Per tile: load S_j, mask (causal by absolute position, keys past the context),
//                 exchange the row max through shared memory, online softmax in base 2 with packed f32x2
//                 arithmetic, write P_j; bf16 writes P as hi + lo bf16 parts (two PV products) so P keeps
//                 fp32 accuracy, as the decode kernel does. The running max only moves when it grows by
//                 more than 2^8 (then the row's O is rescaled in tensor memory), so O and the row sum always
//                 share one reference max and the result is exact; the epilogue divides by the sum and
//                 stores the row, half a row per thread.
// Keys at or past the context end get P = 0; their V rows in a partly filled page tile were never written
// and may hold NaN (0 * NaN = NaN in the MMA), so those rows are zeroed in shared memory and 16-key groups
// wholly past the end are skipped. Every wait is bounded; on a timeout the CTA records
// PKV_DEVERR_WAIT_TIMEOUT, drains its copies and MMAs, frees tensor memory and exits.
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
constexpr int kPfRows = 128;       // GQA-packed rows per CTA = MMA M
constexpr int kPfKeys = 64;        // keys per tile = S MMA N
constexpr int kPfSoftmaxWarp0 = 3; // warps 3..10 run the softmax
constexpr int kPfPvWarp = 11;      // lane 0 issues the P.V MMAs
constexpr int kPfThreads = 12 * 32;
constexpr int kPfRescaleLog2 = 8;  // the reference max moves when a row's max grows by more than 2^8

template <int D>
struct PfConfig {
  static constexpr int kTileBytes = 16 * D * 2;      // one 16-key page tile of K or V
  static constexpr int kKvBytes = kPfKeys * D * 2;   // one 64-key tile of K (or of V)
  // >= 116 KB of shared memory, so one CTA per SM owns all 512 tensor-memory columns
  static constexpr int kStages = D == 256 ? 3 : (D == 128 ? 6 : 8);
  static constexpr int kBarOffset = 2 * kStages * kKvBytes;
  static constexpr int kSmemBytes = kBarOffset + 4096 + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kColQ = D;
  static constexpr uint32_t kColS = D + D / 2;
};

template <typename I>
struct PfArgs {
  const void* query;
  int64_t q_st, q_sh;  // elements
  const int32_t* cu_q;
  const I* tables;
  int64_t table_stride;
  int32_t max_blocks;
  const I* seq_lens;
  int32_t batch, num_pages, block_size;
  int32_t rows_per_page, rows_per_head;
  int32_t num_kv_heads;
  int32_t group_log2;  // log2(G)
  int32_t split_p;     // bf16: P as hi + lo parts (fp32-accurate) instead of one rounded bf16 value
  float scale_log2;
  void* out;
  int64_t o_st, o_sh;  // elements
  int32_t* error_flag;
};

// Shared-memory barriers and flags of one CTA (after the K and V rings).
template <int NST>
struct PfBarriers {
  uint64_t q_ready;
  uint64_t k_full[NST], k_empty[NST], v_full[NST], v_empty[NST];
  uint64_t s_full[2], p_full[2], pv_done[2];
  uint64_t mma_idle;
  uint32_t tmem_base;
  int32_t abort;     // a role gave up on a wait: the others stop at their next step
  int32_t bad_page;
  float xmax[2][2 * kPfRows];  // per tile parity: partial row maxima of the two threads of each row
  float xsum[2 * kPfRows];     // partial row sums for the epilogue
};

template <typename T, typename I, int D>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap, const __grid_constant__ CUtensorMap vmap,
                      const PfArgs<I> a) {
  using Cfg = PfConfig<D>;
  constexpr int NST = Cfg::kStages;
  static_assert(sizeof(PfBarriers<NST>) <= 4096, "barrier block exceeds its shared-memory reservation");
  constexpr bool kBf16 = kSplitP<T>;
  constexpr uint32_t kIdescS = umma_idesc_f16(kBf16, false, kPfRows, kPfKeys);
  constexpr uint32_t kIdescO = umma_idesc_f16(kBf16, true, kPfRows, D);
  const bool split = kBf16 && a.split_p != 0;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint8_t* ks = smem;                                   // NST x [D/64][64 keys][64]
  uint8_t* vs = ks + NST * Cfg::kKvBytes;               // NST x [4 page tiles][D/64][16 keys][64]
  auto* bar = reinterpret_cast<PfBarriers<NST>*>(smem + Cfg::kBarOffset);
  volatile int32_t* abort_flag = &bar->abort;

  const int b = blockIdx.z, kvh = blockIdx.y;
  const int group = 1 << a.group_log2;
  const int tokens = kPfRows >> a.group_log2;  // chunk tokens per CTA
  const int q_begin = a.cu_q[b];
  const int q_len = a.cu_q[b + 1] - q_begin;
  const int t0 = blockIdx.x * tokens;
  if (t0 >= q_len) return;
  int64_t len = load_index(a.seq_lens, b);
  const int64_t cap = static_cast<int64_t>(a.max_blocks) * a.block_size;
  if (len > cap) len = cap;
  const int64_t pos0 = len - q_len;  // absolute position of chunk token 0
  const int ntok = min(tokens, q_len - t0);
  const int64_t last_pos = pos0 + t0 + ntok - 1;
  const int n_tiles = last_pos < 0 ? 0 : static_cast<int>((last_pos + kPfKeys) / kPfKeys);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    mbar_init(&bar->q_ready, 2 * kPfRows);
    for (int s = 0; s < NST; ++s) {
      mbar_init(&bar->k_full[s], 1);
      mbar_init(&bar->k_empty[s], 1);
      mbar_init(&bar->v_full[s], 1);
      mbar_init(&bar->v_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bar->s_full[s], 1);
      mbar_init(&bar->p_full[s], 2 * kPfRows);
      mbar_init(&bar->pv_done[s], 1);
    }
    mbar_init(&bar->mma_idle, 2);  // one arrival per MMA-issuing thread
    bar->abort = 0;
    bar->bad_page = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bar->tmem_base, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar->tmem_base;

  auto give_up = [&]() {
    *abort_flag = 1;
    raise_device_error(a.error_flag, PKV_DEVERR_WAIT_TIMEOUT);
  };

  if (warp == 0 || warp == 2) {
    // ---------------- loads: warp 0 fills the K ring, warp 2 the V ring
    const bool is_k = warp == 0;
    const I* trow = a.tables + static_cast<int64_t>(b) * a.table_stride;
    const int tiles_per_page = a.block_size >> 4;
    const int64_t pages = (len + a.block_size - 1) / a.block_size;
    const uint64_t policy = policy_evict_first();
    uint64_t* full = is_k ? bar->k_full : bar->v_full;
    uint64_t* empty = is_k ? bar->k_empty : bar->v_empty;
    uint8_t* ring = is_k ? ks : vs;
    int issued = 0;  // key tiles whose copies were issued
    for (int j = 0; j < n_tiles; ++j) {
      const int s = j % NST;
      int64_t row = -1;
      bool bad = false;
      if (lane < kPfKeys / 16) {
        const int tile = j * (kPfKeys / 16) + lane;  // 16-key page tile
        const int page_local = tile / tiles_per_page;
        if (page_local < pages) {  // tiles past the context stay unloaded; their keys are masked
          const int64_t page = load_index(trow, page_local);
          if (page < 0 || page >= a.num_pages) {
            bad = true;
          } else {
            row = page * a.rows_per_page + static_cast<int64_t>(kvh) * a.rows_per_head +
                  (tile - page_local * tiles_per_page) * 16;
          }
        }
      }
      if (__any_sync(0xffffffffu, bad) && lane == 0) bar->bad_page = 1;
      const uint32_t bytes = __popc(__ballot_sync(0xffffffffu, row >= 0)) * Cfg::kTileBytes;
      // tile j reuses the stage that S_{j-NST} (K) or PV_{j-NST} (V) read
      int go = 1;
      if (lane == 0) {
        if (j >= NST && !mbar_wait_bounded(&empty[s], ((j / NST) + 1) & 1, kPrefillWaitNs)) {
          give_up();
          go = 0;
        } else if (*abort_flag) {
          go = 0;
        }
        if (go) mbar_arrive_expect_tx(&full[s], bytes);
      }
      if (!__shfl_sync(0xffffffffu, go, 0)) break;
      if (row >= 0) {
        if (is_k) {
          uint8_t* dst = ring + s * Cfg::kKvBytes + lane * 2048;
#pragma unroll
          for (int bx = 0; bx < D / 64; ++bx)
            tma_load_2d(dst + bx * (kPfKeys * 128), &kmap, &full[s], bx * 64, static_cast<int32_t>(row), policy);
        } else {
          tma_load_3d(ring + s * Cfg::kKvBytes + lane * Cfg::kTileBytes, &vmap, &full[s], 0,
                      static_cast<int32_t>(row), 0, policy);
        }
      }
      issued = j + 1;
    }
    if (lane == 0 && *abort_flag) {
      // copies of the last NST issued tiles may still be landing in shared memory: let them finish
      for (int j = max(0, issued - NST); j < issued; ++j)
        mbar_wait_bounded(&full[j % NST], (j / NST) & 1, kPrefillWaitNs);
    }
  } else if (warp == 1 || warp == kPfPvWarp) {
    // ---------------- MMA issue: lane 0 of warp 1 issues S = Q K^T, lane 0 of the last warp O += P V.
    // Each issuer's commits and waits overlap the other's MMAs, so the tensor pipe stays fed.
    if (lane == 0) {
      bool ok = true;
      if (warp == 1) {
        const uint32_t t_q = tmem + Cfg::kColQ, t_s = tmem + Cfg::kColS;
        ok = mbar_wait_bounded(&bar->q_ready, 0, kPrefillWaitNs);
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int s = j % NST;
          // S/P buffer j % 2 is free once PV_{j-2} (the other issuer) has read P_{j-2}
          ok = mbar_wait_bounded(&bar->k_full[s], (j / NST) & 1, kPrefillWaitNs) &&
               (j < 2 || mbar_wait_bounded(&bar->pv_done[j & 1], ((j - 2) >> 1) & 1, kPrefillWaitNs)) &&
               !*abort_flag;
          if (!ok) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(ks + s * Cfg::kKvBytes);
          const uint32_t d = t_s + (j & 1) * kPfKeys;
#pragma unroll
          for (int k = 0; k < D / 16; ++k) {
            const uint32_t ka = k_addr + (k >> 2) * (kPfKeys * 128) + (k & 3) * 32;
            tc_mma_ts(d, t_q + k * 8, umma_desc_sw128(ka, 16, 1024), kIdescS, k > 0);
          }
          tc_commit(&bar->s_full[j & 1]);
          tc_commit(&bar->k_empty[s]);
        }
      } else {
        const uint32_t t_o = tmem, t_s = tmem + Cfg::kColS;
        for (int j = 0; ok && j < n_tiles; ++j) {
          const int s = j % NST;
          ok = mbar_wait_bounded(&bar->v_full[s], (j / NST) & 1, kPrefillWaitNs) &&
               mbar_wait_bounded(&bar->p_full[j & 1], (j >> 1) & 1, kPrefillWaitNs) && !*abort_flag;
          if (!ok) break;
          tc_fence_after();
          const int64_t key0 = static_cast<int64_t>(j) * kPfKeys;
          const int64_t valid = (len - key0 + 15) / 16;  // 16-key groups inside the context
          const int groups = valid < kPfKeys / 16 ? static_cast<int>(valid) : kPfKeys / 16;
          const uint32_t v_addr = smem_u32(vs + s * Cfg::kKvBytes);
          const uint32_t p = t_s + (j & 1) * kPfKeys;
          for (int kk = 0; kk < groups; ++kk)
            tc_mma_ts(t_o, p + kk * 8, umma_desc_sw128(v_addr + kk * Cfg::kTileBytes, 2048, 1024), kIdescO,
                      j > 0 || kk > 0);
          if (split) {
            for (int kk = 0; kk < groups; ++kk)
              tc_mma_ts(t_o, p + kPfKeys / 2 + kk * 8, umma_desc_sw128(v_addr + kk * Cfg::kTileBytes, 2048, 1024),
                        kIdescO, true);
          }
          tc_commit(&bar->pv_done[j & 1]);
          tc_commit(&bar->v_empty[s]);
        }
      }
      if (!ok && !*abort_flag) give_up();
      tc_commit(&bar->mma_idle);  // arrives once every MMA this thread issued has completed
      if (!mbar_wait_bounded(&bar->mma_idle, 0, kPrefillWaitNs)) give_up();
    }
    __syncwarp();
  } else {
    // ---------------- softmax: two threads per row, 32 key columns of each tile apiece
    const int sw = warp - kPfSoftmaxWarp0;
    const int quad = warp & 3;            // this warp's tensor-memory lanes: 32 * quad .. + 31
    const int half = sw >> 2;             // 0: keys 0-31 of a tile (and columns 0 .. D/2 - 1), 1: the rest
    const int r = quad * 32 + lane;
    const int sid = half * kPfRows + r;   // index among the 256 softmax threads
    const int tok = r >> a.group_log2;
    const int head = kvh * group + (r & (group - 1));
    const int64_t qpos = pos0 + t0 + tok;
    const int64_t visible = qpos + 1 < len ? qpos + 1 : len;  // keys [0, visible) are attended
    const uint32_t lane_addr = static_cast<uint32_t>(quad * 32) << 16;
    const uint32_t t_o = tmem + lane_addr + half * (D / 2);
    const uint32_t t_s = tmem + lane_addr + Cfg::kColS;
    const int pair_bar = 1 + quad;        // named barrier of the two warps that share these rows
    const bool valid_tok = tok < ntok;
    // ---- the row's query (this thread's half of it) into tensor memory, two 16-bit values per column
    {
      const uint4* qrow = reinterpret_cast<const uint4*>(static_cast<const T*>(a.query) +
                                                         static_cast<int64_t>(q_begin + t0 + tok) * a.q_st +
                                                         head * a.q_sh + half * (D / 2));
      const uint32_t t_q = tmem + lane_addr + Cfg::kColQ + half * (D / 4);
#pragma unroll
      for (int c = 0; c < D / 64; ++c) {  // 32 elements = 16 columns per step
        uint32_t w[16];
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          const uint4 x = valid_tok ? qrow[c * 4 + v] : make_uint4(0, 0, 0, 0);
          w[4 * v] = x.x;
          w[4 * v + 1] = x.y;
          w[4 * v + 2] = x.z;
          w[4 * v + 3] = x.w;
        }
        tmem_st16(t_q + c * 16, w);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bar->q_ready);
    }
    const uint64_t scale2 = f2_pack(a.scale_log2, a.scale_log2);
    float m_ref = kNegInf, l = 0.f;       // reference max (log2 units) and this half's share of the sum
    // A thread that gives up on a wait stops at the next exchange together with its partner (the exchange
    // barrier has no time limit, so both threads of a row must always reach it).
    bool failed = false;
    for (int j = 0; j < n_tiles; ++j) {
      const uint32_t t_sp = t_s + (j & 1) * kPfKeys;  // this tile's S/P buffer
      const bool mine = !failed &&
                        __all_sync(0xffffffffu, mbar_wait_bounded(&bar->s_full[j & 1], (j >> 1) & 1, kPrefillWaitNs)) &&
                        !__any_sync(0xffffffffu, *abort_flag != 0);
      float sv[32];
      float mx = kNegInf;
      if (mine) {
        tc_fence_after();
        uint32_t raw[32];
        tmem_ld32(t_sp + half * 32, raw);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[i] = __uint_as_float(raw[i]);
        const int64_t lim = visible - (static_cast<int64_t>(j) * kPfKeys + half * 32);  // visible among mine
        if (__any_sync(0xffffffffu, lim < 32)) {
#pragma unroll
          for (int i = 0; i < 32; ++i) sv[i] = i < lim ? sv[i] : kNegInf;
        }
#pragma unroll
        for (int i = 0; i < 32; i += 2) mx = fmax3(mx, sv[i], sv[i + 1]);
      }
      // row max over both halves (scale > 0, so the max of the raw scores is the max of the scaled ones).
      // The barrier also orders both threads' S loads before either overwrites the buffer with P.
      bar->xmax[j & 1][sid] = mx;
      if (!named_barrier_and(pair_bar, 64, mine)) {
        failed = true;
        break;
      }
      mx = fmaxf(mx, bar->xmax[j & 1][sid ^ kPfRows]);
      const float mt = mx * a.scale_log2;
      // reference max: moves on the first tile and whenever the row max grows by more than 2^8; both
      // threads of a row see the same mt, so they decide alike
      const bool grow = mt > m_ref + kPfRescaleLog2;
      if (__any_sync(0xffffffffu, grow)) {
        const float m_new = fmaxf(m_ref, mt);
        const float alpha = m_ref == kNegInf ? 0.f : fast_exp2(m_ref - m_new);
        if (j > 0) {
          // O holds PV_0 .. PV_{j-1}: wait for PV_{j-1}, then scale this half of the row in place
          if (!__all_sync(0xffffffffu,
                          mbar_wait_bounded(&bar->pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, kPrefillWaitNs))) {
            failed = true;
            continue;
          }
          tc_fence_after();
          const uint64_t alpha2 = f2_pack(alpha, alpha);
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; i += 2) {
              const float2 v = f2_unpack(f2_mul(f2_pack(__uint_as_float(o[i]), __uint_as_float(o[i + 1])), alpha2));
              o[i] = __float_as_uint(v.x);
              o[i + 1] = __float_as_uint(v.y);
            }
            tmem_st16(t_o + c * 32, o);
            tmem_st16(t_o + c * 32 + 16, o + 16);
          }
          tmem_st_wait();
        }
        l *= alpha;
        m_ref = m_new;
      }
      const float base = m_ref == kNegInf ? 0.f : m_ref;
      const uint64_t nbase2 = f2_pack(-base, -base);
      uint32_t ph[16], pl[16];
      uint64_t sum2 = f2_pack(0.f, 0.f);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float2 x = f2_unpack(f2_fma(f2_pack(sv[2 * i], sv[2 * i + 1]), scale2, nbase2));
        const float p0 = fast_exp2(x.x), p1 = fast_exp2(x.y);
        const uint64_t p2 = f2_pack(p0, p1);
        sum2 = f2_add(sum2, p2);
        if (split) {
          // hi = p truncated to bf16 (exact in fp32), lo = bf16(p - hi): hi + lo carries p to ~2^-16
          const uint32_t b0 = __float_as_uint(p0) & 0xffff0000u, b1 = __float_as_uint(p1) & 0xffff0000u;
          ph[i] = __byte_perm(b0, b1, 0x7632);
          const float2 lo = f2_unpack(f2_sub(p2, f2_pack(__uint_as_float(b0), __uint_as_float(b1))));
          pl[i] = pack2<T>(lo.x, lo.y);
        } else {
          ph[i] = pack2<T>(p0, p1);
        }
      }
      const float2 s2 = f2_unpack(sum2);
      l += s2.x + s2.y;
      // V rows of never-written slots in the page tile that holds the last key: zero them (P is 0 there,
      // but 0 * NaN would poison O); 16-key groups wholly past the end are not multiplied at all
      const int64_t tail = len - static_cast<int64_t>(j) * kPfKeys;  // keys of this tile inside the context
      if (tail < kPfKeys && (tail & 15) != 0) {
        const int s = j % NST;
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(&bar->v_full[s], (j / NST) & 1, kPrefillWaitNs))) {
          failed = true;
          continue;
        }
        const int first = static_cast<int>(tail & 15), pt = static_cast<int>(tail >> 4);
        uint8_t* tile = vs + s * Cfg::kKvBytes + pt * Cfg::kTileBytes;
        const int chunks = (16 - first) * (D / 8);  // 16-byte chunks of rows first..15 in every 64-column box
        for (int c = sid; c < chunks; c += 2 * kPfRows) {
          const int row = first + c / (D / 8), w = c % (D / 8);
          *reinterpret_cast<uint4*>(tile + (w >> 3) * 2048 + row * 128 + (w & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      // P over the scores: hi of keys 32 * half .. + 31 at columns 16 * half .., lo 32 columns further
      tmem_st16(t_sp + half * 16, ph);
      if (split) tmem_st16(t_sp + kPfKeys / 2 + half * 16, pl);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&bar->p_full[j & 1]);
    }
    if (failed && lane == 0) give_up();
    // ---------------- epilogue: O / l for the rows of this CTA's valid tokens, half a row per thread
    bar->xsum[sid] = l;
    bool ok = named_barrier_and(pair_bar, 64, !failed && !__any_sync(0xffffffffu, *abort_flag != 0));
    if (ok) {
      const float lt = l + bar->xsum[sid ^ kPfRows];
      T* orow = static_cast<T*>(a.out) + static_cast<int64_t>(q_begin + t0 + tok) * a.o_st + head * a.o_sh +
                half * (D / 2);
      if (n_tiles == 0) {
        if (valid_tok)
          for (int c = 0; c < D / 16; ++c) reinterpret_cast<uint4*>(orow)[c] = make_uint4(0, 0, 0, 0);
      } else {
        const int jl = n_tiles - 1;
        ok = __all_sync(0xffffffffu, mbar_wait_bounded(&bar->pv_done[jl & 1], (jl >> 1) & 1, kPrefillWaitNs));
        if (!ok) {
          if (lane == 0) give_up();
        } else {
          tc_fence_after();
          const float inv = lt > 0.f ? 1.f / lt : 0.f;
#pragma unroll 1
          for (int c = 0; c < D / 64; ++c) {
            uint32_t o[32];
            tmem_ld32(t_o + c * 32, o);
            tmem_ld_wait();
            if (valid_tok) {
#pragma unroll
              for (int v = 0; v < 4; ++v) {
                uint4 w;
                w.x = pack2<T>(__uint_as_float(o[8 * v + 0]) * inv, __uint_as_float(o[8 * v + 1]) * inv);
                w.y = pack2<T>(__uint_as_float(o[8 * v + 2]) * inv, __uint_as_float(o[8 * v + 3]) * inv);
                w.z = pack2<T>(__uint_as_float(o[8 * v + 4]) * inv, __uint_as_float(o[8 * v + 5]) * inv);
                w.w = pack2<T>(__uint_as_float(o[8 * v + 6]) * inv, __uint_as_float(o[8 * v + 7]) * inv);
                reinterpret_cast<uint4*>(orow + c * 32)[v] = w;
              }
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (threadIdx.x == 0 && bar->bad_page) raise_device_error(a.error_flag, PKV_DEVERR_PAGE_OUT_OF_RANGE);
  if (warp == 1) tmem_dealloc(tmem, Cfg::kTmemCols);
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
int launch_prefill_tc(const CUtensorMap& km, const CUtensorMap& vm, const PfArgs<I>& a, int64_t max_q_len,
                      cudaStream_t s) {
  using Cfg = PfConfig<D>;
  auto kern = prefill_tc_kernel<T, I, D>;
  const cudaError_t e = prepare_kernel(reinterpret_cast<const void*>(kern), Cfg::kSmemBytes);
  if (e != cudaSuccess) return cuda_status(e, "prefill_tc_kernel smem attribute");
  const int64_t tokens = kPfRows >> a.group_log2;
  const dim3 grid(static_cast<unsigned>((max_q_len + tokens - 1) / tokens), a.num_kv_heads, a.batch);
  kern<<<grid, kPfThreads, Cfg::kSmemBytes, s>>>(km, vm, a);
  return cuda_status(cudaGetLastError(), "prefill_tc_kernel launch");
}

template <typename I>
int run_prefill(const void* query, int64_t q_st, int64_t q_sh, const int32_t* cu_q, int64_t total_q,
                int64_t max_q_len, const void* kpool, const void* vpool, int64_t num_pages, int64_t num_kv_heads,
                int64_t block_size, int64_t head_dim, int64_t sp, int64_t sh, int64_t ss, const void* tables,
                int64_t table_stride, int64_t max_blocks, const void* seq_lens, int64_t batch, int64_t num_q_heads,
                float scale, void* out, int64_t o_st, int64_t o_sh, int dtype, int flags, int32_t* error_flag,
                cudaStream_t stream) {
  const int64_t group = num_q_heads / num_kv_heads;
  const float scale_log2 = scale * kLog2e;
  const uintptr_t align = reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(kpool) |
                          reinterpret_cast<uintptr_t>(vpool) | reinterpret_cast<uintptr_t>(out);
  const int64_t rows = (num_pages - 1) * (sp / head_dim) + (num_kv_heads - 1) * (sh / head_dim) + block_size;
  int group_log2 = 0;
  while ((1ll << group_log2) < group) ++group_log2;
  const bool tc_ok = (dtype == PKV_DTYPE_F16 || dtype == PKV_DTYPE_BF16) && scale > 0.f &&
                     (head_dim == 64 || head_dim == 128 || head_dim == 256) && (1ll << group_log2) == group &&
                     group <= 16 && block_size % 16 == 0 && ss == head_dim && sp % head_dim == 0 &&
                     sh % head_dim == 0 && q_st % 8 == 0 && q_sh % 8 == 0 && o_st % 8 == 0 && o_sh % 8 == 0 &&
                     align % 16 == 0 && rows < (1ll << 31) && total_q < (1ll << 31) && batch < 65536 &&
                     num_kv_heads < 65536;
  bump_stat(kStatPrefill);
  if (tc_ok) {
    CUtensorMap km, vm;
    // K: pool rows of head_dim elements, 64-column x 16-row boxes
    const cuuint64_t kdims[2] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(rows)};
    const cuuint64_t kstr[1] = {static_cast<cuuint64_t>(head_dim * 2)};
    const cuuint32_t kbox[2] = {64, 16};
    int st = encode(&km, kpool, dtype, 2, kdims, kstr, kbox);
    if (st != PKV_OK) return st;
    // V: (64 columns, rows, head_dim / 64), one 16-row page tile per box
    const cuuint64_t vdims[3] = {64, static_cast<cuuint64_t>(rows), static_cast<cuuint64_t>(head_dim / 64)};
    const cuuint64_t vstr[2] = {static_cast<cuuint64_t>(head_dim * 2), 128};
    const cuuint32_t vbox[3] = {64, 16, static_cast<cuuint32_t>(head_dim / 64)};
    st = encode(&vm, vpool, dtype, 3, vdims, vstr, vbox);
    if (st != PKV_OK) return st;
    PfArgs<I> a{query, q_st, q_sh, cu_q, static_cast<const I*>(tables), table_stride, static_cast<int32_t>(max_blocks),
                static_cast<const I*>(seq_lens), static_cast<int32_t>(batch), static_cast<int32_t>(num_pages),
                static_cast<int32_t>(block_size), static_cast<int32_t>(sp / head_dim),
                static_cast<int32_t>(sh / head_dim), static_cast<int32_t>(num_kv_heads), group_log2,
                (flags & PKV_PREFILL_ROUND_PROBS) ? 0 : 1, scale_log2, out, o_st, o_sh, error_flag};
    if (dtype == PKV_DTYPE_F16) {
      if (head_dim == 64) return launch_prefill_tc<__half, I, 64>(km, vm, a, max_q_len, stream);
      if (head_dim == 128) return launch_prefill_tc<__half, I, 128>(km, vm, a, max_q_len, stream);
      return launch_prefill_tc<__half, I, 256>(km, vm, a, max_q_len, stream);
    }
    if (head_dim == 64) return launch_prefill_tc<__nv_bfloat16, I, 64>(km, vm, a, max_q_len, stream);
    if (head_dim == 128) return launch_prefill_tc<__nv_bfloat16, I, 128>(km, vm, a, max_q_len, stream);
    return launch_prefill_tc<__nv_bfloat16, I, 256>(km, vm, a, max_q_len, stream);
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

extern "C" int pkv_paged_prefill_ex(const void* query, int64_t q_stride_token, int64_t q_stride_head,
                                    const int32_t* cu_q, int64_t total_q, int64_t max_q_len, const void* key_pool,
                                    const void* value_pool, int64_t num_pages, int64_t num_kv_heads,
                                    int64_t block_size, int64_t head_dim, int64_t stride_page, int64_t stride_head,
                                    int64_t stride_slot, const void* block_tables, int64_t table_stride,
                                    int64_t max_blocks, const void* seq_lens, int index_dtype, int64_t batch,
                                    int64_t num_q_heads, float scale, void* output, int64_t o_stride_token,
                                    int64_t o_stride_head, int dtype, int flags, int32_t* error_flag, void* stream) {
  clear_error();
  PKV_REQUIRE(dtype_size(dtype) > 0, "paged_prefill: unsupported dtype %d", dtype);
  PKV_REQUIRE(index_dtype == PKV_INDEX_I32 || index_dtype == PKV_INDEX_I64, "paged_prefill: bad index dtype");
  PKV_REQUIRE((flags & ~PKV_PREFILL_ROUND_PROBS) == 0, "paged_prefill: unknown flags 0x%x", flags);
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
                                o_stride_token, o_stride_head, dtype, flags, error_flag, s);
  return run_prefill<int64_t>(query, q_stride_token, q_stride_head, cu_q, total_q, max_q_len, key_pool, value_pool,
                              num_pages, num_kv_heads, block_size, head_dim, stride_page, stride_head, stride_slot,
                              block_tables, table_stride, max_blocks, seq_lens, batch, num_q_heads, scale, output,
                              o_stride_token, o_stride_head, dtype, flags, error_flag, s);
}

extern "C" int pkv_paged_prefill(const void* query, int64_t q_stride_token, int64_t q_stride_head, const int32_t* cu_q,
                                 int64_t total_q, int64_t max_q_len, const void* key_pool, const void* value_pool,
                                 int64_t num_pages, int64_t num_kv_heads, int64_t block_size, int64_t head_dim,
                                 int64_t stride_page, int64_t stride_head, int64_t stride_slot,
                                 const void* block_tables, int64_t table_stride, int64_t max_blocks,
                                 const void* seq_lens, int index_dtype, int64_t batch, int64_t num_q_heads,
                                 float scale, void* output, int64_t o_stride_token, int64_t o_stride_head, int dtype,
                                 int32_t* error_flag, void* stream) {
  return pkv_paged_prefill_ex(query, q_stride_token, q_stride_head, cu_q, total_q, max_q_len, key_pool, value_pool,
                              num_pages, num_kv_heads, block_size, head_dim, stride_page, stride_head, stride_slot,
                              block_tables, table_stride, max_blocks, seq_lens, index_dtype, batch, num_q_heads, scale,
                              output, o_stride_token, o_stride_head, dtype, 0, error_flag, stream);
}
