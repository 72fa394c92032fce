// Ragged causal prefill attention over the paged KV cache on the 5th-generation
// tensor cores (tcgen05 + TMEM), sm_100a.
//
// One CTA = (sequence b, kv head hk, block of QB query tokens) and all G query
// heads that share hk: 256 query rows = two M = 128 tiles (A and B), row
// rho = g * QB + tau for query head hk * G + g and token tau of the block
// (QB = 256 / G; G = 4 gives two heads x 64 tokens per tile).  Every K/V stage
// (128 keys) is loaded once and used by both tiles, and the two tiles
// ping-pong: the tensor core works on one tile's MMAs while the other tile's
// softmax runs.
//
//   warps 0-3 softmax A, warps 4-7 softmax B: thread r of a group owns row r
//             of its tile (TMEM lane r): tcgen05.ld of its 128 scores, causal /
//             validity mask, base-2 online softmax with a lazy O rescale (only
//             when the row max grew by more than 2^8), P (16-bit) written with
//             tcgen05.st over the upper 64 columns of its S buffer -- the P V
//             MMA takes A from tensor memory -- and at the end its O row read
//             back, divided by the row sum and stored;
//   warp 8    producer: K/V stages of 128 keys as two 64-key TMA halves
//             (pages from block_tables[b], 128-byte swizzle) into a
//             kStages-deep ring; it starts as soon as the CTA knows its
//             sequence, without waiting for the TMEM allocation;
//   warp 9    MMA issuer (one thread): S_X = Q_X K^T as two N = 64 halves,
//             O_X += P_X V.  P_X(j) lives in the upper half of S_X's columns,
//             so as soon as P_X(j) is written the thread issues P_X(j) V_j and
//             the lower half of S_X(j+1); the upper half follows once P_X(j) V_j
//             has finished.  The softmax starts on the lower half meanwhile.
//
// TMEM (512 columns, one CTA per SM): S_A [0,128) | S_B [128,256) | O_A | O_B.
// Shared memory: two 128-key K/V stages (D = 128; three at D = 64) and the
// two Q tiles, written by the softmax threads in the 128-byte swizzle.  Key
// rows a stage does not hold (past the context, or pages with an invalid block
// id) are masked in S and their V rows are zeroed before the P V MMA, so stale
// or NaN bytes never reach O -- the reference's masked_fill of V
// (src/inferkernellab/attention.py:301-305).  Semantics are those of the
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

constexpr int kFaTiles = 2;                       // query tiles per CTA
constexpr int kFaKeys = 2 * kKvTile;              // keys per K/V stage
constexpr int kFaProducerWarp = 8;
constexpr int kFaMmaWarp = 9;
constexpr int kFaThreads = 10 * 32;
constexpr int kFaTmemCols = 512;
constexpr float kLazyRescale = 8.0f;  // log2 units: rescale O only when the max grows by 2^8

template <int D>
struct FaShape {
  static constexpr int kRegions = D / 64;                 // 128-byte column regions
  static constexpr int kHalfBytes = kKvTile * D * 2;      // 64 keys of K (or V)
  static constexpr int kStageBytes = 4 * kHalfBytes;      // K halves 0, 1 | V halves 0, 1
  static constexpr int kStages = D >= 128 ? 2 : 3;
  static constexpr int kQTileBytes = kTcRows * D * 2;
  static constexpr int kQRegionBytes = kTcRows * 128;     // 16 KB
  static constexpr int kHalfRegionBytes = kKvTile * 128;  // 8 KB
  static constexpr int kOCol = kFaTiles * kFaKeys;        // O_X at kOCol + X * D
};

struct FaSmem {
  int stages_off, q_off, bars_off, mask_off, flags_off, table_off, scan_off, total;
};

template <int D>
__host__ __device__ inline FaSmem fa_smem_layout() {
  using S = FaShape<D>;
  FaSmem L;
  int off = 0;
  L.stages_off = off;
  off += S::kStages * S::kStageBytes;
  L.q_off = off;
  off += kFaTiles * S::kQTileBytes;
  L.bars_off = off;
  // full, empty per stage; s_full0, s_full1, p_full, pv_done, q_full per tile; mma_idle
  off += (2 * S::kStages + 5 * kFaTiles + 1) * 8;
  L.mask_off = off;
  off += S::kStages * 2 * 8;
  L.flags_off = off;
  off += 16;  // abort flag, TMEM address
  L.table_off = off;
  off += kTableWindow * 4;
  L.scan_off = off;
  off += (kFaThreads / 32 + 6) * 4 + 16;  // warp totals, found sequence, its start / end
  L.total = off;
  return L;
}

// Query tokens per CTA for `group` query heads per kv head.
__host__ __device__ inline int fa_query_block(int group) { return (kFaTiles * kTcRows) / group; }

// A bounded wait whose outcome every lane of the warp shares: the warp-wide
// operations after it (tcgen05.ld / st, the producer's warp reductions) then
// never run with part of the warp gone after a timeout or an abort.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint32_t* err, uint32_t code) {
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, abort_flag, err, code));
}

template <typename E, int D>
__global__ void __launch_bounds__(kFaThreads, 1)
    paged_prefill_tc_kernel(const __grid_constant__ CUtensorMap kmap,
                            const __grid_constant__ CUtensorMap vmap,
                            const __grid_constant__ CUtensorMap qmap,
                            const __grid_constant__ CUtensorMap omap, const PrefillParams p) {
  using S = FaShape<D>;
  using T = typename E::T;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const FaSmem L = fa_smem_layout<D>();
  uint8_t* q_s = smem + L.q_off;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L.bars_off);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* s_full0 = empty_bar + kStages;  // [tile]: keys 0-63 of S_X(j) written
  uint64_t* s_full1 = s_full0 + kFaTiles;   // [tile]: keys 64-127 of S_X(j) written
  uint64_t* p_full = s_full1 + kFaTiles;    // [tile]: P_X(j) written (and V rows zeroed)
  uint64_t* pv_done = p_full + kFaTiles;   // [tile]: P_X(j) V(j) finished
  uint64_t* q_full = pv_done + kFaTiles;   // [tile]: Q_X in shared memory
  uint64_t* mma_idle = q_full + kFaTiles;
  uint64_t* stage_mask = reinterpret_cast<uint64_t*>(smem + L.mask_off);  // 2 per stage
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.flags_off);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L.flags_off + 4);
  int* table_s = reinterpret_cast<int*>(smem + L.table_off);
  int* scan_s = reinterpret_cast<int*>(smem + L.scan_off);
  int* found_s = scan_s + kFaThreads / 32;  // [0] sequence, [1] block, [2] first row, [3] rows
  long long* found_se = reinterpret_cast<long long*>(  // [0] query_starts[b], [1] context_lens[b]
      (reinterpret_cast<uintptr_t>(found_s + 6) + 7) & ~static_cast<uintptr_t>(7));

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = p.num_seqs;
  const int G = p.group;
  const int QB = fa_query_block(G);
  // blockIdx.x = item * num_kv_heads + kv head: every kv head of an item is
  // dispatched together, and items run heaviest first within a sequence.
  const int Hkv = p.num_kv_heads;
  const int hk = static_cast<int>(blockIdx.x % static_cast<unsigned>(Hkv));
  const int item = static_cast<int>(blockIdx.x / static_cast<unsigned>(Hkv));
  const long long cap = static_cast<long long>(p.table_width) * p.src.block_size;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 2);   // one arrive.expect_tx per 64-key half
      mbar_init(&empty_bar[s], 1);  // one tcgen05.commit per consumed stage
    }
    for (int x = 0; x < kFaTiles; ++x) {
      mbar_init(&s_full0[x], 1);
      mbar_init(&s_full1[x], 1);
      mbar_init(&p_full[x], kTcRows);
      mbar_init(&pv_done[x], 1);
      mbar_init(&q_full[x], 1);  // the producer's arrive.expect_tx for the Q box
    }
    mbar_init(mma_idle, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  // Launched with programmatic stream serialization: the CTA may start while
  // the previous kernel on the stream (typically the KV append of the same
  // batch) finishes.  Nothing above touches global memory; griddepcontrol.wait
  // returns once that kernel has completed and its writes are visible.  The
  // early CTA return below counts as the trigger for the next kernel.
  asm volatile("griddepcontrol.wait;" ::: "memory");

  // ---- which (sequence, query block) this CTA owns ----
  int b = 0, qb = 0;
  long long q_row0 = 0;               // packed: first query row of sequence b
  long long q_rows = p.max_query_len;  // query rows of sequence b that exist
  long long start_b = 0, end_b = 0;
  if (!p.packed) {
    const int blocks = (p.max_query_len + QB - 1) / QB;
    b = item / blocks;
    qb = blocks - 1 - (item - b * blocks);  // heaviest block of each sequence first
    start_b = load_index(p.starts, b, p.index64);
    end_b = load_index(p.ends, b, p.index64);
    __syncthreads();  // the barrier initialisation above is visible to every warp
  } else {
    // Sequences in chunks of one per thread: block prefix sums until the chunk
    // holding block index blockIdx.x is found.
    const int x = item;
    int base = 0;
    if (tid == 0) found_s[0] = -1;
    for (int c0 = 0; c0 < B; c0 += kFaThreads) {
      const int i = c0 + tid;
      int n = 0, cu0 = 0, len = 0;
      long long st = 0, en = 0;
      if (i < B) {  // this sequence's metadata, all loads in one round trip
        cu0 = p.cu_seqlens[i];
        len = p.cu_seqlens[i + 1] - cu0;
        st = load_index(p.starts, i, p.index64);
        en = load_index(p.ends, i, p.index64);
        n = len > 0 ? (len + QB - 1) / QB : 0;
      }
      int chunk_total = 0;
      const int before = base + block_exclusive_scan<kFaThreads>(n, scan_s, &chunk_total);
      if (n > 0 && x >= before && x < before + n) {
        found_s[0] = i;
        found_s[1] = n - 1 - (x - before);  // heaviest block of each sequence first
        found_s[2] = cu0;
        found_s[3] = len;
        found_se[0] = st;
        found_se[1] = en;
      }
      base += chunk_total;
      __syncthreads();
      if (found_s[0] >= 0) break;  // CTA-uniform
    }
    if (found_s[0] < 0) return;  // CTA-uniform, before TMEM is allocated
    b = found_s[0];
    qb = found_s[1];
    q_row0 = found_s[2];
    q_rows = found_s[3];
    start_b = found_se[0];
    end_b = found_se[1];
  }
  const long long t0 = static_cast<long long>(qb) * QB;

  // Row r of tile x <-> (query head hk * G + g, token t): the Q tile is one TMA
  // box {64 elements, HT heads, 128 / HT tokens}, so row r = token * HT + head.
  // G >= 2: tile x holds heads x * HT .. x * HT + HT - 1 (HT = G / 2) and the
  // block's QB = 128 / HT tokens; G = 1: tile x holds tokens x * 128 .. + 127.
  const int lg_ht = G >= 2 ? __ffs(G) - 2 : 0;
  const int HT = 1 << lg_ht;
  auto tile_row = [&](int x, int row, int& g, long long& t) {
    if (G >= 2) {
      g = x * HT + (row & (HT - 1));
      t = t0 + (row >> lg_ht);
    } else {
      g = 0;
      t = t0 + x * kTcRows + row;
    }
  };
  constexpr int kChunks = D / 8;                      // 16-byte chunks per row
  constexpr int kCopies = kTcRows * kChunks / kTcRows;  // epilogue chunks per softmax thread
  const int x_tile = warp >> 2;

  // ---- TMEM: 512 columns, allocated by the MMA warp; the producer warp does
  // not wait for it (named barrier 1 spans the other nine warps) ----
  uint32_t tmem = 0;
  if (warp != kFaProducerWarp) {
    if (warp == kFaMmaWarp) {
      tc::tmem_alloc(tmem_slot, kFaTmemCols);
      tc::tmem_relinquish();
    }
    tc::fence_before_sync();
    asm volatile("bar.sync 1, %0;" ::"n"(kFaThreads - 32) : "memory");
    tc::fence_after_sync();
    tmem = *tmem_slot;
  }

  long long len_b = end_b - start_b;
  if (start_b < 0 || len_b <= 0) len_b = 0;
  const long long key_end = end_b < cap ? end_b : cap;  // real keys are < key_end
  const long long rows_here = p.packed ? len_b : p.max_query_len;
  long long kmax = 0;
  if (t0 < len_b) kmax = start_b + min(t0 + QB, len_b);
  if (!p.packed && t0 + QB > len_b && t0 < rows_here && kmax < 1) kmax = 1;  // padding rows
  if (kmax > key_end) kmax = key_end;
  const int n_kt = static_cast<int>((kmax + kFaKeys - 1) / kFaKeys);

  if (warp == kFaProducerWarp) {
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
    // The two Q tiles: one box per 64-element region (rows past the tensor are
    // zero-filled; rows of other sequences are never stored).
    if (lane == 0 && n_kt > 0) {
      tma_prefetch_desc(&qmap);
#pragma unroll
      for (int x = 0; x < kFaTiles; ++x) {
        const int head0 = hk * G + (G >= 2 ? x * HT : 0);
        const long long tok0 = t0 + (G >= 2 ? 0 : x * kTcRows);
        mbar_arrive_expect_tx(&q_full[x], static_cast<uint32_t>(S::kQTileBytes));
#pragma unroll
        for (int c = 0; c < S::kRegions; ++c) {
          uint8_t* dst = q_s + x * S::kQTileBytes + c * S::kQRegionBytes;
          if (p.packed)
            tma_load_3d(dst, &qmap, &q_full[x], c * 64, head0, static_cast<int>(q_row0 + tok0));
          else
            tma_load_4d(dst, &qmap, &q_full[x], c * 64, head0, static_cast<int>(tok0), b);
        }
      }
    }
    __syncwarp();
    int issued = 0;
    for (int it = 0; it < n_kt; ++it) {
      const int s = it % kStages;
      const uint32_t k = static_cast<uint32_t>(it / kStages);
      if (!warp_wait(&empty_bar[s], (k & 1u) ^ 1u, abort_flag, p.err, kErrWaitEmpty))
        break;
      uint8_t* stage = smem + L.stages_off + s * S::kStageBytes;
      const int tok0 = it * kFaKeys;
      const int n0 = static_cast<int>(min(static_cast<long long>(kKvTile), key_end - tok0));
      issue_kv_tile<D>(&kmap, &vmap, p.src, win, b, row_pages, hk, tok0, n0, stage,
                       stage + 2 * S::kHalfBytes, &full_bar[s], &stage_mask[2 * s], p.err, lane);
      const long long rest = key_end - tok0 - kKvTile;
      if (rest > 0) {
        const int n1 = static_cast<int>(min(static_cast<long long>(kKvTile), rest));
        issue_kv_tile<D>(&kmap, &vmap, p.src, win, b, row_pages, hk, tok0 + kKvTile, n1,
                         stage + S::kHalfBytes, stage + 3 * S::kHalfBytes, &full_bar[s],
                         &stage_mask[2 * s + 1], p.err, lane);
      } else if (lane == 0) {
        stage_mask[2 * s + 1] = 0;
        mbar_arrive(&full_bar[s]);  // the second half holds no key
      }
      __syncwarp();
      ++issued;
    }
    if (lane == 0) {
      drain_stages<kStages>(full_bar, issued, p.err);
      // ... and the Q boxes (every TMA copy lands before the CTA exits).
      for (int x = 0; x < kFaTiles && n_kt > 0; ++x) drain_stages<1>(&q_full[x], 1, p.err);
    }
  } else if (warp == kFaMmaWarp) {
    // ------------------------------ MMA issuer -----------------------------
    if (lane == 0 && n_kt > 0) {
      const uint32_t id_s = tc::idesc_f16(kTcRows, kKvTile, E::kIsBf16, false, false);
      const uint32_t id_o = tc::idesc_f16(kTcRows, D, E::kIsBf16, false, true);
      const uint32_t q0 = smem_u32(q_s);
      const uint32_t st0 = smem_u32(smem + L.stages_off);
      // S_X(j), keys of half hf (64 keys) -> S_X columns [64 hf, 64 hf + 64).
      auto issue_s = [&](int x, int j, int hf) {
        const uint32_t kb = st0 + (j % kStages) * S::kStageBytes + hf * S::kHalfBytes;
        const uint32_t qx = q0 + x * S::kQTileBytes;
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t reg = static_cast<uint32_t>(k >> 2), kk = static_cast<uint32_t>(k & 3);
          tc::mma_f16(tmem + x * kFaKeys + hf * kKvTile,
                      tc::sdesc_sw128(qx + reg * S::kQRegionBytes + kk * 32, 16, 1024),
                      tc::sdesc_sw128(kb + reg * S::kHalfRegionBytes + kk * 32, 16, 1024), id_s,
                      k > 0);
        }
        tc::commit(hf == 0 ? &s_full0[x] : &s_full1[x]);
      };
      // O_X += P_X(j) V_j: P_X in S_X's columns [64, 128), 16 keys per MMA.
      auto issue_pv = [&](int x, int j) {
        const uint32_t vb = st0 + (j % kStages) * S::kStageBytes + 2 * S::kHalfBytes;
#pragma unroll
        for (int k = 0; k < kFaKeys / 16; ++k)
          tc::mma_f16_tmem_a(tmem + S::kOCol + x * D, tmem + x * kFaKeys + kKvTile + k * 8,
                             tc::sdesc_sw128(vb + (k >> 2) * S::kHalfBytes + (k & 3) * 2048,
                                             S::kHalfRegionBytes, 1024),
                             id_o, j > 0 || k > 0);
        tc::commit(&pv_done[x]);
      };
      auto wait = [&](uint64_t* bar, uint32_t parity) {
        return mbar_wait_bounded(bar, parity, abort_flag, p.err, kErrWaitFull);
      };
      bool ok = wait(&full_bar[0], 0);
      for (int x = 0; x < kFaTiles && ok; ++x) {
        ok = wait(&q_full[x], 0);
        if (!ok) break;
        tc::fence_after_sync();
        issue_s(x, 0, 0);
        issue_s(x, 0, 1);
      }
      for (int j = 0; j < n_kt && ok; ++j) {
        const uint32_t ph = static_cast<uint32_t>(j & 1);
        for (int x = 0; x < kFaTiles && ok; ++x) {
          ok = wait(&p_full[x], ph);
          if (!ok) break;
          tc::fence_after_sync();
          issue_pv(x, j);
          if (x == kFaTiles - 1) tc::commit(&empty_bar[j % kStages]);
          if (j + 1 < n_kt) {
            // Keys 0-63 of S_X(j+1) go to columns P_X(j) does not use: at once.
            ok = wait(&full_bar[(j + 1) % kStages], static_cast<uint32_t>(((j + 1) / kStages) & 1));
            if (!ok) break;
            tc::fence_after_sync();
            issue_s(x, j + 1, 0);
            // Keys 64-127 overwrite P_X(j): only once P_X(j) V_j has finished.
            ok = wait(&pv_done[x], ph);
            if (!ok) break;
            tc::fence_after_sync();
            issue_s(x, j + 1, 1);
          }
        }
      }
      // Every MMA this thread issued has finished before TMEM can be freed.
      tc::commit(mma_idle);
      mbar_wait_bounded(mma_idle, 0, abort_flag, p.err, kErrDrain);
    }
  } else {
    // ------------------------------ softmax ------------------------------
    const int x = x_tile;
    const int r = tid & (kTcRows - 1);  // row of the tile = TMEM lane
    // Keys [0, row_lim(g, t)) are visible to the row of head g, token t.
    auto row_lim = [&](int g, long long t) -> int {
      if (g >= G) return 0;
      if (t < len_b) return static_cast<int>(min(start_b + t + 1, key_end));
      if (!p.packed && t < rows_here) return key_end > 0 ? 1 : 0;  // padding row: key 0 only
      return 0;
    };
    int g_me;
    long long t_me;
    tile_row(x, r, g_me, t_me);
    const int lim = row_lim(g_me, t_me);
    const uint32_t lane_base = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    const uint32_t s_col = static_cast<uint32_t>(x * kFaKeys);
    const uint32_t o_col = static_cast<uint32_t>(S::kOCol + x * D);

    float m_used = -INFINITY;  // max the row's P and O are currently scaled to
    float l_sum = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kt && ok; ++j) {
      const int s = j % kStages;
      const uint32_t ph = static_cast<uint32_t>(j & 1);
      ok = warp_wait(&full_bar[s], (j / kStages) & 1, abort_flag, p.err, kErrWaitFull);
      if (!ok) break;
      tc::fence_after_sync();
      const uint64_t m0 = stage_mask[2 * s], m1 = stage_mask[2 * s + 1];
      const int key0 = j * kFaKeys;
      // Keys [key0, key0 + nv) are visible to this row (causal / context limit).
      // The stage holds keys [0, kh); a page inside them with an invalid block
      // id clears its bits in the stage mask ("holes", stage-uniform, rare).
      const int nv = min(max(lim - key0, 0), kFaKeys);
      const int kh = static_cast<int>(min(static_cast<long long>(kFaKeys), key_end - key0));
      const uint64_t want0 = kh >= 64 ? ~0ull : ((1ull << kh) - 1ull);
      const uint64_t want1 = kh >= 128 ? ~0ull : (kh > 64 ? ((1ull << (kh - 64)) - 1ull) : 0ull);
      const bool holes = (m0 & want0) != want0 || (m1 & want1) != want1;
      // The 128 scores in two halves of 64: P of the first half stays packed in
      // registers until the second half's max is known, so that a (rare) lazy
      // rescale in the second half can still rescale it.
      uint32_t pk0[32];
      float o_scale = 1.f;  // factor O must be rescaled by before this stage's P V
#pragma unroll 1
      for (int hf = 0; hf < 2; ++hf) {
        if (!warp_wait(hf == 0 ? &s_full0[x] : &s_full1[x], ph, abort_flag, p.err,
                       kErrWaitFull)) {
          ok = false;
          break;
        }
        tc::fence_after_sync();
        uint32_t sr[kKvTile];
        tc::ld32(lane_base + s_col + hf * 64, *reinterpret_cast<uint32_t(*)[32]>(&sr[0]));
        tc::ld32(lane_base + s_col + hf * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(&sr[32]));
        tc::wait_ld();
        // Raw scores, masked keys set to -inf, and their max (scale > 0, so the
        // max of the scaled scores is the scaled max).
        const int nvh = min(max(nv - hf * 64, 0), 64);
        float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // independent chains
        if (nvh == 64 && !holes) {
#pragma unroll
          for (int c = 0; c < kKvTile; ++c) mx4[c & 3] = fmaxf(mx4[c & 3], __uint_as_float(sr[c]));
        } else {
          uint64_t vm = nvh >= 64 ? ~0ull : ((1ull << nvh) - 1ull);
          if (holes) vm &= hf == 0 ? m0 : m1;
          const uint32_t vlo = static_cast<uint32_t>(vm), vhi = static_cast<uint32_t>(vm >> 32);
#pragma unroll
          for (int c = 0; c < kKvTile; ++c) {
            const bool valid = (((c < 32 ? vlo : vhi) >> (c & 31)) & 1u) != 0u;
            const float v = valid ? __uint_as_float(sr[c]) : -INFINITY;
            sr[c] = __float_as_uint(v);
            mx4[c & 3] = fmaxf(mx4[c & 3], v);
          }
        }
        const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])) * p.scale_log2;
        float alpha = 1.f;
        if (mx != -INFINITY && (m_used == -INFINITY || mx > m_used + kLazyRescale)) {
          if (m_used != -INFINITY) alpha = fast_exp2(m_used - mx);
          m_used = mx;
        }
        if (alpha != 1.f) {
          o_scale *= alpha;
          if (hf == 1) {  // the first half's P was scaled to the old max
#pragma unroll
            for (int c = 0; c < 32; ++c) pk0[c] = scale_pack2<E>(pk0[c], alpha);
          }
        }
        // P = 2^(s * scale_log2 - m): masked keys (-inf) give 0; a row with no
        // visible key so far (m = -inf) subtracts 0 and gets only zeros.
        const float msub = m_used == -INFINITY ? 0.f : m_used;
        float ps4[4] = {0.f, 0.f, 0.f, 0.f};
        uint32_t pk[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const float e0 = fast_exp2(fmaf(__uint_as_float(sr[2 * c]), p.scale_log2, -msub));
          const float e1 = fast_exp2(fmaf(__uint_as_float(sr[2 * c + 1]), p.scale_log2, -msub));
          ps4[(2 * c) & 3] += e0;
          ps4[(2 * c + 1) & 3] += e1;
          pk[c] = pack2<E>(e0, e1);
        }
        l_sum = l_sum * alpha + ((ps4[0] + ps4[1]) + (ps4[2] + ps4[3]));
        if (hf == 0) {
#pragma unroll
          for (int c = 0; c < 32; ++c) pk0[c] = pk[c];
        } else {
          // P row -> columns [64, 128) of this tile's S buffer (A operand in TMEM).
          tc::st32(lane_base + s_col + 64, pk0);
          tc::st32(lane_base + s_col + 96, pk);
        }
      }
      if (!ok) break;
      const bool rescale = o_scale != 1.f;

      // O_X is rescaled only when a row of this warp raised its max by more
      // than 2^8 (rare); only then must P V of the previous stage be complete.
      if (__any_sync(0xffffffffu, rescale)) {
        ok = warp_wait(&pv_done[x], ph ^ 1u, abort_flag, p.err, kErrWaitFull);
        if (!ok) break;
        tc::fence_after_sync();
        const float a = o_scale;
#pragma unroll
        for (int cb = 0; cb < D / 32; ++cb) {
          uint32_t o[32];
          tc::ld32(lane_base + o_col + cb * 32, o);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * a);
          tc::st32(lane_base + o_col + cb * 32, o);
        }
      }
      // Tile A zeroes the V rows of keys the stage does not hold (stage-uniform
      // test); tile B's P V is issued after tile A's, so it sees them too.
      if (x == 0 && (m0 & m1) != ~0ull) {
        uint8_t* vst = smem + L.stages_off + s * S::kStageBytes + 2 * S::kHalfBytes;
        for (int e = r; e < kFaKeys * S::kRegions; e += kTcRows) {
          const int key = e & (kFaKeys - 1);
          const int reg = e / kFaKeys;
          if (!(((key < 64 ? m0 : m1) >> (key & 63)) & 1ull)) {
            uint8_t* vrow = vst + (key >> 6) * S::kHalfBytes + reg * S::kHalfRegionBytes +
                            (key & 63) * 128;
#pragma unroll
            for (int c = 0; c < 8; ++c) reinterpret_cast<uint4*>(vrow)[c] = make_uint4(0, 0, 0, 0);
          }
        }
      }
      tc::wait_st();
      tc::fence_proxy_async_smem();  // zeroed V rows (generic stores) -> the MMA
      tc::fence_before_sync();
      mbar_arrive(&p_full[x]);
    }
    // The last P V done (it completes after every earlier MMA of the tile).
    const bool have_o =
        ok && n_kt > 0 &&
        warp_wait(&pv_done[x], static_cast<uint32_t>((n_kt - 1) & 1), abort_flag, p.err,
                  kErrWaitFull);
    // O row / l -> this tile's Q buffer (free: every S MMA has finished) in the
    // Q box's layout (row r, 128-byte swizzle).  A tile whose rows all have
    // output leaves as TMA stores of that box (one thread, asynchronous); the
    // others are copied out by the tile's threads, coalesced, row by row.
    uint8_t* stg = q_s + x * S::kQTileBytes;
    if (have_o) {
      tc::fence_after_sync();
      const float inv = 1.f / l_sum;
#pragma unroll
      for (int cb = 0; cb < D / 32; ++cb) {
        uint32_t o[32];
        tc::ld32(lane_base + o_col + cb * 32, o);
        tc::wait_ld();
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint4 v;
          v.x = pack2<E>(__uint_as_float(o[8 * c + 0]) * inv, __uint_as_float(o[8 * c + 1]) * inv);
          v.y = pack2<E>(__uint_as_float(o[8 * c + 2]) * inv, __uint_as_float(o[8 * c + 3]) * inv);
          v.z = pack2<E>(__uint_as_float(o[8 * c + 4]) * inv, __uint_as_float(o[8 * c + 5]) * inv);
          v.w = pack2<E>(__uint_as_float(o[8 * c + 6]) * inv, __uint_as_float(o[8 * c + 7]) * inv);
          const int chunk = cb * 4 + c;
          *reinterpret_cast<uint4*>(stg + (chunk >> 3) * S::kQRegionBytes +
                                    tc::sw128_offset(r, chunk & 7)) = v;
        }
      }
      tc::fence_proxy_async_smem();  // the staged rows -> the TMA store
    }
    // Every thread of the tile reaches this barrier, whatever happened above;
    // the rows are copied out only when all 128 were staged.
    uint32_t all_staged;
    asm volatile(
        "{\n\t.reg .pred q, a;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred a, %2, %3, q;\n\t"
        "selp.u32 %0, 1, 0, a;\n\t}"
        : "=r"(all_staged)
        : "r"(have_o ? 1u : 0u), "r"(2 + x), "n"(kTcRows)
        : "memory");
    // Rows with output: tokens below len_b (packed), or below the padded width
    // when the context is not empty (padding rows attend key 0).
    const long long valid_end = key_end <= 0 ? 0 : (p.packed ? len_b : max(len_b, rows_here));
    const long long tile_t0 = t0 + (G >= 2 ? 0 : x * kTcRows);
    const int tile_tokens = G >= 2 ? (kTcRows >> lg_ht) : kTcRows;
    const bool tile_full = G >= 2 ? tile_t0 + tile_tokens <= valid_end && G == 2 * HT
                                  : tile_t0 + tile_tokens <= valid_end;
    if (all_staged && tile_full) {
      if (r == 0) {
        const int head0 = hk * G + (G >= 2 ? x * HT : 0);
#pragma unroll
        for (int c = 0; c < S::kRegions; ++c) {
          if (p.packed)
            tma_store_3d(&omap, stg + c * S::kQRegionBytes, c * 64, head0,
                         static_cast<int>(q_row0 + tile_t0));
          else
            tma_store_4d(&omap, stg + c * S::kQRegionBytes, c * 64, head0,
                         static_cast<int>(tile_t0), b);
        }
        bulk_commit_group();
        bulk_wait_group_read0();  // the staging buffer is read before the CTA exits
      }
    } else if (all_staged) {
#pragma unroll 4
      for (int it = 0; it < kCopies; ++it) {
        const int idx = it * kTcRows + r;
        const int row = idx / kChunks, c = idx % kChunks;
        int g;
        long long t;
        tile_row(x, row, g, t);
        if (row_lim(g, t) > 0) {
          const int h = hk * G + g;
          T* base = reinterpret_cast<T*>(p.out);
          T* orow = p.packed ? base + (q_row0 + t) * p.o_stride_token + h * p.o_stride_head
                             : base + b * p.o_stride_seq + h * p.o_stride_head + t * p.o_stride_token;
          reinterpret_cast<uint4*>(orow)[c] = *reinterpret_cast<const uint4*>(
              stg + (c >> 3) * S::kQRegionBytes + tc::sw128_offset(row, c & 7));
        }
      }
    }
  }

  // ---- teardown: every TMEM access is done, the MMA warp frees TMEM ----
  tc::fence_before_sync();
  __syncthreads();
  // The next kernel on the stream may now be scheduled: triggering only here,
  // at the end of each CTA, keeps its CTAs from taking SM slots that this
  // kernel's later CTAs still need.
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == kFaMmaWarp) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tmem, kFaTmemCols);
  }
}

template <typename E, int D>
int launch_tc_t(const CUtensorMap& kmap, const CUtensorMap& vmap, const CUtensorMap& qmap,
                const CUtensorMap& omap, const PrefillParams& p, dim3 grid, cudaStream_t stream) {
  // Over half of the SM's shared memory, so one CTA (512 TMEM columns) per SM.
  const int smem = std::max(fa_smem_layout<D>().total + 1024, 116 * 1024);
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
  cfg.blockDim = dim3(kFaThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t lerr = cudaLaunchKernelEx(&cfg, kern, kmap, vmap, qmap, omap, p);
  if (lerr != cudaSuccess) return cuda_status(lerr, "paged_prefill_tc_kernel launch");
  return cuda_status(cudaGetLastError(), "paged_prefill_tc_kernel launch");
}

}  // namespace

int prefill_tc_query_block(int group) { return fa_query_block(group); }

int prefill_tc_query_heads_per_tile(int group) { return group >= 2 ? group / 2 : 1; }

int launch_prefill_tc(const CUtensorMap& kmap, const CUtensorMap& vmap, const CUtensorMap& qmap,
                      const CUtensorMap& omap, const PrefillParams& p, int head_dim, bool bf16,
                      unsigned grid_x, unsigned grid_y, cudaStream_t stream) {
  const dim3 grid(grid_x, grid_y);
  if (head_dim == 128)
    return bf16 ? launch_tc_t<BF16, 128>(kmap, vmap, qmap, omap, p, grid, stream)
                : launch_tc_t<Half, 128>(kmap, vmap, qmap, omap, p, grid, stream);
  if (head_dim == 64)
    return bf16 ? launch_tc_t<BF16, 64>(kmap, vmap, qmap, omap, p, grid, stream)
                : launch_tc_t<Half, 64>(kmap, vmap, qmap, omap, p, grid, stream);
  return set_error(B200_ERR_UNSUPPORTED, "tcgen05 prefill supports head_dim 64 and 128");
}

}  // namespace b200
