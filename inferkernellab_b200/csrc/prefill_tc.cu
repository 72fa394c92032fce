// Ragged causal prefill attention over the paged KV cache on the 5th-generation
// tensor cores (tcgen05 + TMEM), sm_100a.
//
// One CTA = (sequence b, query head h, tile of 128 query tokens): the 128 rows
// are the M dimension of every MMA and row r lives in TMEM lane r.
//
//   warp 4  producer   streams 64-token K/V tiles of kv head h / G through a
//                      kStages-deep ring with TMA (pages from block_tables[b],
//                      128-byte swizzle), exactly as the mma.sync kernel does;
//   warp 5  MMA issuer (one thread) S_j = Q K_j^T into one of two TMEM score
//                      buffers, then O += P_j V_j into the TMEM accumulator;
//                      S_{j+1} is issued before P_j V_j so the tensor core
//                      works on the next scores while the softmax runs;
//   warps 0-3 softmax  thread r owns query row r: it loads its 64 scores with
//                      tcgen05.ld, applies the causal / validity mask and a
//                      base-2 online softmax, rescales its O row in TMEM when
//                      its running max grew by more than 2^8 (lazy rescale),
//                      and writes its P row (16-bit, tcgen05.st) over the first
//                      32 columns of the S buffer it just read: the P V MMA
//                      takes A from tensor memory.  At the end it reads its O
//                      row, divides by the row sum and stores it.
//
// Operand layouts (tcgen05.cuh): Q is K-major SW128 (written by the softmax
// threads), K is K-major SW128 and V is MN-major SW128 as TMA writes them, P is
// in TMEM.  Shared memory is Q + two K/V stages (D = 128) or three (D = 64),
// about 100 KB, so two CTAs share an SM and one's softmax overlaps the other's
// MMAs; TMEM is 256 columns per CTA (S0 | S1 | O), two CTAs fill the SM's 512.  Key rows a tile does not hold (past the context, or pages with an
// invalid block id) are masked in S and their V rows are zeroed before the
// P V MMA, so stale or NaN bytes never reach O -- the reference's masked_fill
// of V (src/inferkernellab/attention.py:301-305).  Semantics are those of the
// mma.sync kernel in prefill.cu (reference attention.py:230-321).
//
// Every mbarrier wait is bounded (1 s); on a timeout the CTA raises its abort
// flag, records the error bit, waits (bounded) for its own MMAs and TMA copies
// to finish and frees its TMEM before it exits.
#include <math.h>

#include <algorithm>

#include "../../include/b200_paged_attn.h"
#include "attn_core.cuh"
#include "common.cuh"
#include "host_common.h"
#include "prefill_params.h"
#include "tcgen05.cuh"

namespace b200 {

namespace {

constexpr int kTcSoftmaxWarps = 4;
constexpr int kTcProducerWarp = 4;
constexpr int kTcMmaWarp = 5;
constexpr int kTcThreads = 6 * 32;
constexpr int kTcTmemCols = 256;  // S0 [0,64) | S1 [64,128) | O [128, 128 + D)
constexpr int kTcOCol = 128;
constexpr float kLazyRescale = 8.0f;  // log2 units: rescale O only when the max grows by 2^8

template <int D>
struct TcShape {
  static constexpr int kRegions = D / 64;               // 128-byte column regions
  static constexpr int kTileBytes = kKvTile * D * 2;    // K (or V) of one 64-token tile
  static constexpr int kQBytes = kTcRows * D * 2;       // 128 query rows
  static constexpr int kStages = D >= 128 ? 2 : 3;
  static constexpr int kQRegionBytes = kTcRows * 128;    // 16 KB
  static constexpr int kKvRegionBytes = kKvTile * 128;   // 8 KB
};

struct TcSmem {
  int stages_off, q_off, bars_off, mask_off, flags_off, table_off, begin_off, total;
};

template <int D>
__host__ __device__ inline TcSmem tc_smem_layout(int num_seqs, int packed) {
  using S = TcShape<D>;
  TcSmem L;
  int off = 0;
  L.stages_off = off;
  off += S::kStages * 2 * S::kTileBytes;
  L.q_off = off;
  off += S::kQBytes;
  L.bars_off = off;
  off += (2 * S::kStages + 10) * 8;  // full, empty, s_full[2], s_free[2], p_full[2], q_full,
                                     // idle, pv_done[2]
  L.mask_off = off;
  off += S::kStages * 8;
  L.flags_off = off;
  off += 16;  // abort flag, TMEM address
  L.table_off = off;
  off += kTableWindow * 4;
  L.begin_off = off;
  if (packed) off += (num_seqs + 1) * 4 + (kTcThreads / 32) * 4;
  L.total = off;
  return L;
}

template <typename E, int D>
__global__ void __launch_bounds__(kTcThreads, 2)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  using S = TcShape<D>;
  using T = typename E::T;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const TcSmem L = tc_smem_layout<D>(p.num_seqs, p.packed);
  uint8_t* q_s = smem + L.q_off;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L.bars_off);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* s_full = empty_bar + kStages;
  uint64_t* s_free = s_full + 2;
  // [2]: P of the tile in S buffer (tile & 1) written.  One barrier per buffer:
  // the softmax may write P of tile j + 1 before the MMA thread has taken P of
  // tile j, but P of tile j + 2 only after P V of tile j (S_{j+2} waits for it),
  // so each barrier has at most one phase outstanding.
  uint64_t* p_full = s_free + 2;
  uint64_t* q_full = p_full + 2;
  uint64_t* mma_idle = q_full + 1;
  uint64_t* pv_done = mma_idle + 1;  // [2]: P V of a tile in S buffer (tile & 1) finished
  uint64_t* stage_mask = reinterpret_cast<uint64_t*>(smem + L.mask_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.flags_off);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.flags_off + 4);
  int* table_s = reinterpret_cast<int*>(smem + L.table_off);
  int* begin_s = reinterpret_cast<int*>(smem + L.begin_off);
  int* scan_s = begin_s + p.num_seqs + 1;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = p.num_seqs;
  const int h = blockIdx.y;
  const int hkv = h / p.group;
  const long long cap = static_cast<long long>(p.table_width) * p.src.block_size;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);  // one tcgen05.commit per consumed tile
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], kTcSoftmaxWarps * 32);
    }
    mbar_init(&p_full[0], kTcSoftmaxWarps * 32);
    mbar_init(&p_full[1], kTcSoftmaxWarps * 32);
    mbar_init(q_full, kTcSoftmaxWarps * 32);
    mbar_init(mma_idle, 1);
    mbar_init(&pv_done[0], 1);
    mbar_init(&pv_done[1], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Launched with programmatic stream serialization: the CTA may start while
  // the previous kernel on the stream (typically the KV append of the same
  // batch) finishes.  Nothing above touches global memory; griddepcontrol.wait
  // returns once that kernel has completed and its writes are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  // ---- which (sequence, 128-row query tile) this CTA owns ----
  int b = 0, qt = 0;
  if (!p.packed) {
    const int tiles = (p.max_query_len + kTcRows - 1) / kTcRows;
    b = blockIdx.x / tiles;
    qt = tiles - 1 - (blockIdx.x - b * tiles);  // heaviest tile of each sequence first
  } else {
    const int chunk = (B + kTcThreads - 1) / kTcThreads;
    const int lo = min(B, tid * chunk);
    const int hi = min(B, lo + chunk);
    int sum = 0;
    for (int i = lo; i < hi; ++i) {
      const long long n = p.cu_seqlens[i + 1] - p.cu_seqlens[i];
      sum += n > 0 ? static_cast<int>((n + kTcRows - 1) / kTcRows) : 0;
    }
    int total_tiles = 0;
    int acc = block_exclusive_scan<kTcThreads>(sum, scan_s, &total_tiles);
    for (int i = lo; i < hi; ++i) {
      begin_s[i] = acc;
      const long long n = p.cu_seqlens[i + 1] - p.cu_seqlens[i];
      acc += n > 0 ? static_cast<int>((n + kTcRows - 1) / kTcRows) : 0;
    }
    if (tid == 0) begin_s[B] = total_tiles;
    __syncthreads();
    const int x = blockIdx.x;
    if (x >= begin_s[B]) return;  // CTA-uniform, before TMEM is allocated
    int lo2 = 0, hi2 = B;
    while (hi2 - lo2 > 1) {
      const int mid = (lo2 + hi2) >> 1;
      if (begin_s[mid] <= x) lo2 = mid; else hi2 = mid;
    }
    b = lo2;
    const int tiles = begin_s[b + 1] - begin_s[b];
    qt = tiles - 1 - (x - begin_s[b]);
  }

  // ---- TMEM: 256 columns, allocated by the MMA warp ----
  if (warp == kTcMmaWarp) {
    tc::tmem_alloc(tmem_slot, kTcTmemCols);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;

  const long long start_b = load_index(p.starts, b, p.index64);
  const long long end_b = load_index(p.ends, b, p.index64);
  long long len_b = end_b - start_b;
  if (start_b < 0 || len_b <= 0) len_b = 0;
  const long long key_end = end_b < cap ? end_b : cap;  // real keys are < key_end
  const int t0 = qt * kTcRows;
  const long long rows_here = p.packed ? len_b : p.max_query_len;
  long long kmax = 0;
  if (t0 < len_b) kmax = start_b + min(static_cast<long long>(t0 + kTcRows), len_b);
  if (!p.packed && t0 + kTcRows > len_b && t0 < rows_here && kmax < 1) kmax = 1;
  if (kmax > key_end) kmax = key_end;
  const int n_ktiles = static_cast<int>((kmax + kKvTile - 1) / kKvTile);

  if (warp == kTcProducerWarp) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      tma_prefetch_desc(&kmap);
      tma_prefetch_desc(&vmap);
    }
    TableWindow win;
    win.ids = table_s;
    win.row = -1;
    win.first = 0;
    win.count = 0;
    const int row_pages = static_cast<int>((key_end + p.src.block_size - 1) / p.src.block_size);
    int issued = 0;
    for (int it = 0; it < n_ktiles; ++it) {
      const int s = it % kStages;
      const uint32_t k = static_cast<uint32_t>(it / kStages);
      if (!mbar_wait_bounded(&empty_bar[s], (k & 1u) ^ 1u, abort_flag, p.err, kErrWaitEmpty))
        break;
      const int tok0 = it * kKvTile;
      const int ntok = static_cast<int>(min(static_cast<long long>(kKvTile), key_end - tok0));
      uint8_t* kdst = smem + L.stages_off + s * 2 * S::kTileBytes;
      issue_kv_tile<D>(&kmap, &vmap, p.src, win, b, row_pages, hkv, tok0, ntok, kdst,
                       kdst + S::kTileBytes, &full_bar[s], &stage_mask[s], p.err, lane);
      ++issued;
    }
    if (lane == 0) drain_stages<kStages>(full_bar, issued, p.err);
  } else if (warp == kTcMmaWarp) {
    // ------------------------------ MMA issuer -----------------------------
    if (lane == 0 && n_ktiles > 0) {
      const uint32_t id_s = tc::idesc_f16(kTcRows, kKvTile, E::kIsBf16, false, false);
      const uint32_t id_o = tc::idesc_f16(kTcRows, D, E::kIsBf16, false, true);
      const uint32_t q0 = smem_u32(q_s);
      const uint32_t st0 = smem_u32(smem + L.stages_off);
      bool ok = mbar_wait_bounded(q_full, 0, abort_flag, p.err, kErrWaitFull);
      // Issue whichever is ready first: S_ns (K tile landed, its S buffer free:
      // the softmax has read S_{ns-2} and P V_{ns-2} has consumed P_{ns-2}) or
      // P V_np (its probabilities are written).  Every barrier probed here has
      // at most one phase outstanding, so the parity probes cannot alias.
      int ns = 0, np = 0;  // next S tile, next P V tile
      unsigned long long last = global_timer_ns();
      while (ok && np < n_ktiles) {
        bool progressed = false;
        if (np < ns && mbar_test_wait(&p_full[np & 1], (np >> 1) & 1)) {
          tc::fence_after_sync();
          const int s = np % kStages;
          const uint32_t vb = st0 + s * 2 * S::kTileBytes + S::kTileBytes;
          const uint32_t p_tmem = tmem + (np & 1) * kKvTile;  // P_np over S_np's columns
#pragma unroll
          for (int k = 0; k < kKvTile / 16; ++k)
            tc::mma_f16_tmem_a(tmem + kTcOCol, p_tmem + k * 8,
                               tc::sdesc_sw128(vb + k * 2048, S::kKvRegionBytes, 1024), id_o,
                               np > 0 || k > 0);
          tc::commit(&pv_done[np & 1]);
          tc::commit(&empty_bar[s]);
          ++np;
          progressed = true;
        }
        if (ns < n_ktiles && ns <= np + 1) {
          const int s = ns % kStages;
          const bool ready =
              mbar_test_wait(&full_bar[s], (ns / kStages) & 1) &&
              (ns < 2 || (mbar_test_wait(&s_free[ns & 1], ((ns - 2) >> 1) & 1) &&
                          mbar_test_wait(&pv_done[ns & 1], ((ns - 2) >> 1) & 1)));
          if (ready) {
            tc::fence_after_sync();
            const uint32_t kb = st0 + s * 2 * S::kTileBytes;
            const uint32_t d_s = tmem + (ns & 1) * kKvTile;
#pragma unroll
            for (int k = 0; k < D / 16; ++k) {
              const uint32_t reg = static_cast<uint32_t>(k >> 2), kk = static_cast<uint32_t>(k & 3);
              tc::mma_f16(d_s, tc::sdesc_sw128(q0 + reg * S::kQRegionBytes + kk * 32, 16, 1024),
                          tc::sdesc_sw128(kb + reg * S::kKvRegionBytes + kk * 32, 16, 1024), id_s,
                          k > 0);
            }
            tc::commit(&s_full[ns & 1]);
            ++ns;
            progressed = true;
          }
        }
        if (progressed) {
          last = global_timer_ns();
        } else if (*abort_flag) {
          ok = false;
        } else if (global_timer_ns() - last > kWaitLimitNs) {
          *abort_flag = 1;
          if (p.err) atomicOr(p.err, kErrWaitFull);
          ok = false;
        }
      }
      // Every MMA this thread issued has finished before TMEM can be freed.
      tc::commit(mma_idle);
      mbar_wait_bounded(mma_idle, 0, abort_flag, p.err, kErrDrain);
    }
  } else {
    // ------------------------------ softmax ------------------------------
    const int r = tid;  // query row = TMEM lane
    const long long t = t0 + r;
    int lim = 0;  // keys [0, lim) are visible to this row
    if (t < len_b)
      lim = static_cast<int>(min(start_b + t + 1, key_end));
    else if (!p.packed && t < rows_here)
      lim = key_end > 0 ? 1 : 0;  // padding row: key 0 only
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);

    // Q row -> shared memory (K-major SW128), zeros for rows without a query.
    {
      const T* qrow = nullptr;
      if (lim > 0) {
        const T* base = reinterpret_cast<const T*>(p.q);
        qrow = p.packed ? base + (p.cu_seqlens[b] + t) * p.q_stride_token + h * p.q_stride_head
                        : base + b * p.q_stride_seq + h * p.q_stride_head + t * p.q_stride_token;
      }
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        const uint4 v = qrow ? reinterpret_cast<const uint4*>(qrow)[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(q_s + (c >> 3) * S::kQRegionBytes + tc::sw128_offset(r, c & 7)) =
            v;
      }
      tc::fence_proxy_async_smem();
      mbar_arrive(q_full);
    }

    float m_used = -INFINITY;  // max the row's P and O are currently scaled to
    float l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < n_ktiles && ok; ++j) {
      const int s = j % kStages;
      ok = mbar_wait_bounded(&full_bar[s], (j / kStages) & 1, abort_flag, p.err, kErrWaitFull) &&
           mbar_wait_bounded(&s_full[j & 1], (j >> 1) & 1, abort_flag, p.err, kErrWaitFull);
      if (!ok) break;
      tc::fence_after_sync();
      uint32_t sr[kKvTile];
      tc::ld32(lane_base + (j & 1) * kKvTile, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
      tc::ld32(lane_base + (j & 1) * kKvTile + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
      tc::wait_ld();
      tc::fence_before_sync();
      mbar_arrive(&s_free[j & 1]);

      const uint64_t tmask = stage_mask[s];
      const int key0 = j * kKvTile;
      // Keys [key0, key0 + nv) are visible to this row (causal / context limit);
      // the page-validity bits only matter on tiles with holes (tile-uniform).
      const int nv = min(max(lim - key0, 0), kKvTile);
      const uint32_t mlo = static_cast<uint32_t>(tmask);
      const uint32_t mhi = static_cast<uint32_t>(tmask >> 32);
      const bool holes = (mlo & mhi) != 0xffffffffu;
      float x[kKvTile];
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // independent chains
#pragma unroll
      for (int c = 0; c < kKvTile; ++c) {
        bool valid = c < nv;
        if (holes) valid = valid && (((c < 32 ? mlo : mhi) >> (c & 31)) & 1u);
        x[c] = valid ? __uint_as_float(sr[c]) * p.scale_log2 : -INFINITY;
        mx4[c & 3] = fmaxf(mx4[c & 3], x[c]);
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      float alpha = 1.f;
      bool rescale = false;
      if (mx != -INFINITY && (m_used == -INFINITY || mx > m_used + kLazyRescale)) {
        if (m_used != -INFINITY) {
          alpha = fast_exp2(m_used - mx);
          rescale = true;
        }
        m_used = mx;
      }
      float ps4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < kKvTile; ++c) {
        x[c] = x[c] == -INFINITY ? 0.f : fast_exp2(x[c] - m_used);
        ps4[c & 3] += x[c];
      }
      l_sum = l_sum * alpha + ((ps4[0] + ps4[1]) + (ps4[2] + ps4[3]));

      // O is rescaled only when a row of this warp raised its max by more than
      // 2^8 (rare); only then must P V of the previous tile be complete first.
      // P_j needs no wait: it goes into the S buffer of tile j - 2, whose P V
      // finished before S_j could be issued.  The wait uses the per-buffer
      // pv_done barrier: S_j has been read, so P V of tile j - 2 is done and
      // pv_done[(j - 1) & 1] has at most one phase outstanding.
      if (__any_sync(0xffffffffu, rescale)) {
        ok = mbar_wait_bounded(&pv_done[(j - 1) & 1], ((j - 1) >> 1) & 1, abort_flag, p.err,
                               kErrWaitFull);
        if (!ok) break;
        tc::fence_after_sync();
        const float a = rescale ? alpha : 1.f;
#pragma unroll
        for (int cb = 0; cb < D / 32; ++cb) {
          uint32_t o[32];
          tc::ld32(lane_base + kTcOCol + cb * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * a);
          tc::st32(lane_base + kTcOCol + cb * 32, o);
        }
        tc::wait_st();
      }
      // Zero the V rows of keys this tile does not hold (tile-uniform test).
      if (tmask != ~0ull) {
        const int key = r & (kKvTile - 1);
        const int reg = r >> 6;
        if (reg < S::kRegions && !((tmask >> key) & 1ull)) {
          uint8_t* vrow = smem + L.stages_off + s * 2 * S::kTileBytes + S::kTileBytes +
                          reg * S::kKvRegionBytes + key * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) reinterpret_cast<uint4*>(vrow)[c] = make_uint4(0, 0, 0, 0);
        }
      }
      // P row -> the first 32 columns of this tile's S buffer (A operand in TMEM).
      {
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) pk[c] = pack2<E>(x[2 * c], x[2 * c + 1]);
        tc::st32(lane_base + (j & 1) * kKvTile, pk);
        tc::wait_st();
      }
      tc::fence_proxy_async_smem();  // zeroed V rows (generic stores) -> the MMA
      tc::fence_before_sync();
      mbar_arrive(&p_full[j & 1]);
    }
    // The last P V done (it completes after every earlier MMA of the thread).
    if (ok && n_ktiles > 0 &&
        mbar_wait_bounded(&pv_done[(n_ktiles - 1) & 1], ((n_ktiles - 1) >> 1) & 1, abort_flag,
                          p.err, kErrWaitFull)) {
      tc::fence_after_sync();
      const float inv = 1.f / l_sum;
      T* orow = nullptr;
      if (lim > 0) {
        T* base = reinterpret_cast<T*>(p.out);
        orow = p.packed ? base + (p.cu_seqlens[b] + t) * p.o_stride_token + h * p.o_stride_head
                        : base + b * p.o_stride_seq + h * p.o_stride_head + t * p.o_stride_token;
      }
#pragma unroll
      for (int cb = 0; cb < D / 32; ++cb) {
        uint32_t o[32];
        tc::ld32(lane_base + kTcOCol + cb * 32, o);
        tc::wait_ld();
        if (orow) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            uint4 v;
            v.x = pack2<E>(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
            v.y = pack2<E>(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
            v.z = pack2<E>(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
            v.w = pack2<E>(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
            reinterpret_cast<uint4*>(orow + cb * 32)[c] = v;
          }
        }
      }
    }
  }

  // ---- teardown: every TMEM access is done, the MMA warp frees TMEM ----
  tc::fence_before_sync();
  __syncthreads();
  if (warp == kTcMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kTcTmemCols);
  }
}

template <typename E, int D>
int launch_tc_t(const CUtensorMap& kmap, const CUtensorMap& vmap, const PrefillParams& p,
                dim3 grid, cudaStream_t stream) {
  // At least 76 KB, so that no more than two CTAs (2 x 256 TMEM columns) share an SM.
  const int smem = std::max(tc_smem_layout<D>(p.num_seqs, p.packed).total + 1024, 76 * 1024);
  auto kern = paged_prefill_tc_kernel<E, D>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && configured[dev] < smem) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return cuda_status(err, "cudaFuncSetAttribute(prefill tcgen05 smem)");
    configured[dev] = smem;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kTcThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t lerr = cudaLaunchKernelEx(&cfg, kern, kmap, vmap, p);
  if (lerr != cudaSuccess) return cuda_status(lerr, "paged_prefill_tc_kernel launch");
  return cuda_status(cudaGetLastError(), "paged_prefill_tc_kernel launch");
}

}  // namespace

int launch_prefill_tc(const CUtensorMap& kmap, const CUtensorMap& vmap, const PrefillParams& p,
                      int head_dim, bool bf16, unsigned grid_x, unsigned grid_y,
                      cudaStream_t stream) {
  const dim3 grid(grid_x, grid_y);
  if (head_dim == 128)
    return bf16 ? launch_tc_t<BF16, 128>(kmap, vmap, p, grid, stream)
                : launch_tc_t<Half, 128>(kmap, vmap, p, grid, stream);
  if (head_dim == 64)
    return bf16 ? launch_tc_t<BF16, 64>(kmap, vmap, p, grid, stream)
                : launch_tc_t<Half, 64>(kmap, vmap, p, grid, stream);
  return set_error(B200_ERR_UNSUPPORTED, "tcgen05 prefill supports head_dim 64 and 128");
}

}  // namespace b200
