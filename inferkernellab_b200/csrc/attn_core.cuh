// Building blocks shared by the paged decode and paged prefill kernels.
//
//   KvTileShape<D>   -- shared-memory geometry of one 64-token K/V tile as TMA
//                       writes it: `chunks` column regions of 64 rows x
//                       chunk_bytes, each 1024-byte aligned, optionally swizzled.
//   TableWindow      -- producer-private shared-memory copy of part of a
//                       block-table row (one coalesced refill per window).
//   issue_kv_tile()  -- producer side: block ids, validity mask, expect-tx and
//                       the TMA loads of one tile (one warp).
//   block_exclusive_scan() -- warp-shuffle prefix sum over a CTA.
//   load_q_frag()    -- 16 query rows x D as mma.sync A fragments.
//   attend16()       -- consumer side: S = Q K^T for 16 keys, masking, base-2
//                       online softmax and O += P V on mma.sync m16n8k16.
#pragma once

#include "common.cuh"

namespace b200 {

constexpr int kKvTile = 64;  // tokens per pipeline stage

template <int D>
struct KvTileShape {
  static constexpr int kRowBytes = D * 2;
  static constexpr int kChunkBytes = kRowBytes < 128 ? kRowBytes : 128;
  static constexpr int kChunkElems = kChunkBytes / 2;
  static constexpr int kChunks = kRowBytes / kChunkBytes;
  static constexpr int kRegionBytes = kKvTile * kChunkBytes;
  static constexpr int kTileBytes = kKvTile * kRowBytes;  // K (or V) of one tile
};

// Geometry of the paged source, identical for K and V.
struct PagedSource {
  const void* tables;      // block tables
  long long table_stride;  // elements between rows
  long long layer_slot_base;
  int table64;
  int num_blocks;
  int block_size;  // power of two
  int box_rows;    // tokens per TMA box = min(block_size, 64)
};

// Producer-private window of one block-table row, kept in shared memory.  The
// producer walks the pages of a request in order (and revisits them for the
// next kv head), so one coalesced refill per window replaces a dependent
// global load per tile on the TMA issue path.  Entries outside [0, num_blocks)
// are stored as -1.
constexpr int kTableWindow = 512;

struct TableWindow {
  int* ids;   // kTableWindow entries in shared memory
  int row;    // table row held, -1 = none
  int first;  // first page held
  int count;  // pages held
};

// kWide: a window of more than 128 pages is loaded with every load issued
// before any is stored -- one L2/HBM round trip, not one per 128 pages -- at the
// cost of 16 live registers per lane and a longer code path; shorter windows
// always take the 128-page loop.  Decode asks for it (its long rows wait on this
// refill before their first TMA); the prefill kernels do not.
template <bool kWide = false>
__device__ __forceinline__ void table_window_refill(TableWindow& w, const PagedSource& src,
                                                    int row, int first_page, int row_pages,
                                                    uint32_t* err, int lane) {
  const int count = min(kTableWindow, row_pages - first_page);
  const long long base = static_cast<long long>(row) * src.table_stride + first_page;
  auto put = [&](int i, long long v) {
    const bool ok = v >= 0 && v < src.num_blocks;
    if (!ok && err) atomicOr(err, kErrBadBlock);
    w.ids[i] = ok ? static_cast<int>(v) : -1;
  };
  __syncwarp();
  if (kWide && count > 128) {
    constexpr int kPer = kTableWindow / 32;
    long long v[kPer];
#pragma unroll
    for (int u = 0; u < kPer; ++u) {
      const int i = u * 32 + lane;
      v[u] = i < count ? load_index(src.tables, base + i, src.table64) : 0;
    }
#pragma unroll
    for (int u = 0; u < kPer; ++u)
      if (u * 32 + lane < count) put(u * 32 + lane, v[u]);
  } else {
    for (int i0 = 0; i0 < count; i0 += 128) {
      long long v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * 32 + lane;
        v[u] = i < count ? load_index(src.tables, base + i, src.table64) : 0;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u * 32 + lane < count) put(i0 + u * 32 + lane, v[u]);
    }
  }
  __syncwarp();
  w.row = row;
  w.first = first_page;
  w.count = count;
}

// Producer (whole warp): load logical tokens tok0 .. tok0+ntok-1 (ntok <= 64) of
// table row `row` and kv head `head` into stage buffers kdst/vdst, arm `bar`,
// and return the token-validity mask (bit i = tile row i holds a real token).
// Pages whose block id is outside [0, num_blocks) are not loaded and masked.
// `row_pages` = pages of the row that hold tokens (never read past them).
template <int D, bool kWide = false>
__device__ __forceinline__ void issue_kv_tile(const CUtensorMap* kmap, const CUtensorMap* vmap,
                                              const PagedSource& src, TableWindow& win, int row,
                                              int row_pages, int head, int tok0, int ntok,
                                              uint8_t* kdst, uint8_t* vdst, uint64_t* bar,
                                              uint64_t* mask_out, uint32_t* err, int lane) {
  using S = KvTileShape<D>;
  const int rows = src.box_rows;
  const int boxes = kKvTile / rows;
  const uint32_t box_bytes = static_cast<uint32_t>(rows) * S::kChunkBytes;
  const int first_page = tok0 / src.block_size;
  const int last_page = (tok0 + ntok - 1) / src.block_size;
  if (win.row != row || first_page < win.first || last_page >= win.first + win.count)
    table_window_refill<kWide>(win, src, row, first_page, row_pages, err, lane);
  uint32_t mlo = 0, mhi = 0, nvalid = 0;
  for (int j0 = 0; j0 < boxes; j0 += 32) {
    const int j = j0 + lane;
    bool ok = false;
    if (j < boxes && j * rows < ntok) {
      const int pos = tok0 + j * rows;
      ok = win.ids[pos / src.block_size - win.first] >= 0;
    }
    uint64_t m = 0;
    if (ok) {
      const int r0 = j * rows;
      const int r1 = min(ntok, r0 + rows);
      const uint64_t span = (r1 - r0) >= 64 ? ~0ull : ((1ull << (r1 - r0)) - 1ull);
      m = span << r0;
    }
    mlo |= __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(m));
    mhi |= __reduce_or_sync(0xffffffffu, static_cast<uint32_t>(m >> 32));
    nvalid += __popc(__ballot_sync(0xffffffffu, ok));
  }
  if (lane == 0) {
    *mask_out = (static_cast<uint64_t>(mhi) << 32) | mlo;
    mbar_arrive_expect_tx(bar, nvalid * box_bytes * S::kChunks * 2u);
  }
  __syncwarp();
  for (int j0 = 0; j0 < boxes; j0 += 32) {
    const int j = j0 + lane;
    if (j < boxes && j * rows < ntok) {
      const int pos = tok0 + j * rows;
      const int blk = win.ids[pos / src.block_size - win.first];
      if (blk >= 0) {
        const int z = static_cast<int>(src.layer_slot_base +
                                       static_cast<long long>(blk) * src.block_size +
                                       (pos & (src.block_size - 1)));
#pragma unroll
        for (int c = 0; c < S::kChunks; ++c) {
          const int off = c * S::kRegionBytes + j * rows * S::kChunkBytes;
          tma_load_3d(kdst + off, kmap, bar, c * S::kChunkElems, head, z);
          tma_load_3d(vdst + off, vmap, bar, c * S::kChunkElems, head, z);
        }
      }
    }
  }
}

// Producer (whole warp), head-group tiles: tokens tok0 .. tok0+ntok-1 (ntok <=
// tokens = 64 / heads, tok0 a multiple of `tokens`, so one page holds them all)
// of kv heads head0 .. head0+heads-1, one 4-D TMA box per tensor (the map of a
// head-group geometry).  Shared memory receives D / 64 regions of 64 rows x
// 128 bytes, row = head * tokens + token -- the layout issue_kv_tile produces
// for one head and 64 tokens, so the consumers read both alike.  The validity
// mask repeats the token bits once per head.
template <bool kWide = false>
__device__ __forceinline__ void issue_kv_tile_heads(const CUtensorMap* kmap, const CUtensorMap* vmap,
                                                    const PagedSource& src, TableWindow& win,
                                                    int row, int row_pages, int head0, int heads,
                                                    int tok0, int ntok, uint32_t box_bytes,
                                                    uint8_t* kdst, uint8_t* vdst, uint64_t* bar,
                                                    uint64_t* mask_out, uint32_t* err, int lane) {
  const int tokens = kKvTile / heads;
  const int page = tok0 / src.block_size;
  if (win.row != row || page < win.first || page >= win.first + win.count)
    table_window_refill<kWide>(win, src, row, page, row_pages, err, lane);
  if (lane == 0) {
    const int blk = win.ids[page - win.first];
    uint64_t m = 0;
    if (blk >= 0) {
      const uint64_t span = (1ull << ntok) - 1ull;  // ntok <= 32
      for (int h = 0; h < heads; ++h) m |= span << (h * tokens);
    }
    *mask_out = m;
    mbar_arrive_expect_tx(bar, blk >= 0 ? 2u * box_bytes : 0u);
    if (blk >= 0) {
      const int z = static_cast<int>(src.layer_slot_base +
                                     static_cast<long long>(blk) * src.block_size +
                                     (tok0 & (src.block_size - 1)));
      tma_load_4d(kdst, kmap, bar, 0, z, head0, 0);
      tma_load_4d(vdst, vmap, bar, 0, z, head0, 0);
    }
  }
  __syncwarp();
}

// Exclusive prefix sum over the threads of a block of kThreads (a multiple of
// 32): returns the sum of `v` over lower thread ids; *total gets the block sum.
// `warp_tot` is shared scratch of kThreads / 32 ints.  Contains __syncthreads.
template <int kThreads>
__device__ __forceinline__ int block_exclusive_scan(int v, int* warp_tot, int* total) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_tot[warp] = x;
  __syncthreads();
  int before = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kThreads / 32; ++w) {
    const int t = warp_tot[w];
    before += w < warp ? t : 0;
    all += t;
  }
  __syncthreads();
  *total = all;
  return before + x - v;
}

// Bounded wait for the producer's last `kStages` armed phases before exit.
template <int kStages>
__device__ __forceinline__ void drain_stages(uint64_t* full_bar, int issued, uint32_t* err) {
  const int first = issued > kStages ? issued - kStages : 0;
  for (int it = first; it < issued; ++it) {
    const int s = it % kStages;
    const uint32_t k = static_cast<uint32_t>(it / kStages);
    if (mbar_try_wait(&full_bar[s], k & 1u)) continue;
    const unsigned long long t0 = global_timer_ns();
    while (!mbar_try_wait(&full_bar[s], k & 1u)) {
      if (global_timer_ns() - t0 > kWaitLimitNs) {
        if (err) atomicOr(err, kErrDrain);
        return;
      }
    }
  }
}

// A fragments of a 16 x D row block: row r0 = rows[g], r1 = rows[g + 8];
// a null row pointer gives zeros (padding rows).
template <typename E, int D>
__device__ __forceinline__ void load_q_frag(uint32_t (&qf)[D / 16][4], const typename E::T* row0,
                                            const typename E::T* row1, int tq) {
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int c0 = kk * 16 + 2 * tq;
    qf[kk][0] = row0 ? *reinterpret_cast<const uint32_t*>(row0 + c0) : 0u;
    qf[kk][2] = row0 ? *reinterpret_cast<const uint32_t*>(row0 + c0 + 8) : 0u;
    qf[kk][1] = row1 ? *reinterpret_cast<const uint32_t*>(row1 + c0) : 0u;
    qf[kk][3] = row1 ? *reinterpret_cast<const uint32_t*>(row1 + c0 + 8) : 0u;
  }
}

// K and V fragments of 16 keys for mma.sync, held in registers so the stage
// can be released before the math runs.
template <int D>
struct KvFrags {
  uint32_t k[2][D / 16][2];  // per n-tile of 8 keys, per 16-dim k-step: b0, b1
  uint32_t v[D / 8][2];      // per 8-dim n-tile of O: b0 (keys 0-7), b1 (keys 8-15)
};

// Load the fragments of the 16 keys starting at tile row `tok`.  V rows of
// keys that are not real tokens (gmask bit clear) are zeroed so NaN/Inf in
// unwritten slots cannot leak (0 * NaN = NaN); causally masked keys are real
// tokens with finite values by contract and only need P = 0.
template <int D>
__device__ __forceinline__ void load_kv_frags(KvFrags<D>& f, uint32_t kbase, uint32_t vbase,
                                              int tok, uint32_t gmask, uint32_t sw, int lane) {
  using S = KvTileShape<D>;
  const int tq = lane & 3;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    const int trow = tok + nt * 8 + (lane & 7);
    if constexpr (D == 16) {
      const int d = ((lane >> 3) & 1) * 8;
      ldsm_x2(kbase + swizzle_offset(trow * S::kChunkBytes + d * 2, sw), f.k[nt][0][0],
              f.k[nt][0][1]);
    } else {
#pragma unroll
      for (int kk = 0; kk < D / 16; kk += 2) {
        const int d = kk * 16 + (lane >> 3) * 8;
        const int c = d / S::kChunkElems;
        const int dc = d - c * S::kChunkElems;
        ldsm_x4(kbase + c * S::kRegionBytes + swizzle_offset(trow * S::kChunkBytes + dc * 2, sw),
                f.k[nt][kk][0], f.k[nt][kk][1], f.k[nt][kk + 1][0], f.k[nt][kk + 1][1]);
      }
    }
  }
  uint32_t keep0 = 0xffffffffu, keep1 = 0xffffffffu;
  if (gmask != 0xffffu) {
    keep0 = (((gmask >> (2 * tq)) & 1u) ? 0x0000ffffu : 0u) |
            (((gmask >> (2 * tq + 1)) & 1u) ? 0xffff0000u : 0u);
    keep1 = (((gmask >> (2 * tq + 8)) & 1u) ? 0x0000ffffu : 0u) |
            (((gmask >> (2 * tq + 9)) & 1u) ? 0xffff0000u : 0u);
  }
  const int vrow = tok + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
  for (int dt = 0; dt < D / 8; dt += 2) {
    const int d = dt * 8 + (lane >> 4) * 8;
    const int c = d / S::kChunkElems;
    const int dc = d - c * S::kChunkElems;
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(vbase + c * S::kRegionBytes + swizzle_offset(vrow * S::kChunkBytes + dc * 2, sw),
              b0, b1, b2, b3);
    f.v[dt][0] = b0 & keep0;
    f.v[dt][1] = b1 & keep1;
    f.v[dt + 1][0] = b2 & keep0;
    f.v[dt + 1][1] = b3 & keep1;
  }
}

// One 16-key step of attention for a 16-row block held by one warp, from
// fragments in registers.  gmask = validity of the 16 keys (bit i = key i);
// CAUSAL: additionally key (key_pos0 + i) must be < lim0 (row g) / lim1 (row g+8).
template <typename E, int D, bool CAUSAL>
__device__ __forceinline__ void attend16_frags(const uint32_t (&qf)[D / 16][4],
                                               float (&o)[D / 8][4], float (&m_r)[2],
                                               float (&l_r)[2], const KvFrags<D>& f,
                                               uint32_t gmask, int key_pos0, int lim0, int lim1,
                                               float scale_log2, int lane) {
  const int tq = lane & 3;
  float sacc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) mma_16816<E>(sacc[nt], qf[kk], f.k[nt][kk][0], f.k[nt][kk][1]);
  }
  float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int col = nt * 8 + 2 * tq + (e & 1);
      bool valid = (gmask >> col) & 1u;
      if constexpr (CAUSAL) valid = valid && (key_pos0 + col < (e < 2 ? lim0 : lim1));
      sacc[nt][e] = valid ? sacc[nt][e] * scale_log2 : -INFINITY;
    }
    mx0 = fmaxf(mx0, fmaxf(sacc[nt][0], sacc[nt][1]));
    mx1 = fmaxf(mx1, fmaxf(sacc[nt][2], sacc[nt][3]));
  }
  mx0 = quad_max(mx0);
  mx1 = quad_max(mx1);
  const float mn0 = fmaxf(m_r[0], mx0);
  const float mn1 = fmaxf(m_r[1], mx1);
  const float base0 = mn0 == -INFINITY ? 0.f : mn0;
  const float base1 = mn1 == -INFINITY ? 0.f : mn1;
  const float alpha0 = fast_exp2(m_r[0] - base0);
  const float alpha1 = fast_exp2(m_r[1] - base1);
  m_r[0] = mn0;
  m_r[1] = mn1;
  float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    sacc[nt][0] = fast_exp2(sacc[nt][0] - base0);
    sacc[nt][1] = fast_exp2(sacc[nt][1] - base0);
    sacc[nt][2] = fast_exp2(sacc[nt][2] - base1);
    sacc[nt][3] = fast_exp2(sacc[nt][3] - base1);
    ps0 += sacc[nt][0] + sacc[nt][1];
    ps1 += sacc[nt][2] + sacc[nt][3];
  }
  l_r[0] = l_r[0] * alpha0 + ps0;
  l_r[1] = l_r[1] * alpha1 + ps1;
#pragma unroll
  for (int i = 0; i < D / 8; ++i) {
    o[i][0] *= alpha0;
    o[i][1] *= alpha0;
    o[i][2] *= alpha1;
    o[i][3] *= alpha1;
  }
  uint32_t pa[4];
  pa[0] = pack2<E>(sacc[0][0], sacc[0][1]);
  pa[1] = pack2<E>(sacc[0][2], sacc[0][3]);
  pa[2] = pack2<E>(sacc[1][0], sacc[1][1]);
  pa[3] = pack2<E>(sacc[1][2], sacc[1][3]);
#pragma unroll
  for (int dt = 0; dt < D / 8; ++dt) mma_16816<E>(o[dt], pa, f.v[dt][0], f.v[dt][1]);
}

// attend16 straight from shared memory (loads the fragments, then the math).
template <typename E, int D, bool CAUSAL>
__device__ __forceinline__ void attend16(const uint32_t (&qf)[D / 16][4], float (&o)[D / 8][4],
                                         float (&m_r)[2], float (&l_r)[2], uint32_t kbase,
                                         uint32_t vbase, int tok, uint32_t gmask, int key_pos0,
                                         int lim0, int lim1, float scale_log2, uint32_t sw,
                                         int lane) {
  KvFrags<D> f;
  load_kv_frags<D>(f, kbase, vbase, tok, gmask, sw, lane);
  attend16_frags<E, D, CAUSAL>(qf, o, m_r, l_r, f, gmask, key_pos0, lim0, lim1, scale_log2, lane);
}

// ------------------------------------------------------------------------
// Transposed decode step (query group as the MMA N dimension).
//
// For decode, the G query heads that share a KV head are few (G <= 16 here),
// so they become the N = 8 * NT columns of mma.m16n8k16 and the 16 keys of a
// step become the M rows:  S^T[16 keys x 8NT heads] = K[16 x D] . Q^T[D x 8NT],
// O^T[D x 8NT] += V^T[D x 16] . P^T[16 x 8NT].  At G = 4 this needs half the
// MMAs and half the O registers of the heads-as-M form (N pads 4 -> 8, M would
// pad 4 -> 16).  P^T leaves the first MMA in accumulator layout; movmatrix
// transposes its 8x8 halves into the B-operand layout of the second.

// Q^T as B fragments: b0 = Q[head n*8+g][16k + 2t, +1], b1 = ... + 8.
template <typename E, int D, int NT>
__device__ __forceinline__ void load_qT_frag(uint32_t (&qb)[NT][D / 16][2],
                                             const typename E::T* q_group, long long head_stride,
                                             int group, int lane) {
  const int g = lane >> 2;
  const int tq = lane & 3;
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const int head = nt * 8 + g;
    const typename E::T* row = q_group + head * head_stride;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      qb[nt][kk][0] = head < group ? *reinterpret_cast<const uint32_t*>(row + kk * 16 + 2 * tq) : 0u;
      qb[nt][kk][1] =
          head < group ? *reinterpret_cast<const uint32_t*>(row + kk * 16 + 8 + 2 * tq) : 0u;
    }
  }
}

// One 16-key step.  State per thread: m/l for heads (n*8 + 2t, +1) (m is
// uniform over the 8 lanes g; l is this thread's partial over its keys g, g+8),
// oT[n][i] = O^T rows (dims) 16i+g, 16i+g+8 x heads n*8+2t, +1.
template <typename E, int D, int NT>
__device__ __forceinline__ void decode_step16_T(const uint32_t (&qb)[NT][D / 16][2],
                                                float (&oT)[NT][D / 16][4], float (&m)[NT][2],
                                                float (&l)[NT][2], uint32_t kbase, uint32_t vbase,
                                                int tok, uint32_t gmask, float scale_log2,
                                                uint32_t sw, int lane) {
  using S = KvTileShape<D>;
  const int g = lane >> 2;
  const int tq = lane & 3;
  const int mi = lane >> 3;
  uint32_t keep0 = 0xffffffffu, keep1 = 0xffffffffu;
  if (gmask != 0xffffu) {
    keep0 = (((gmask >> (2 * tq)) & 1u) ? 0x0000ffffu : 0u) |
            (((gmask >> (2 * tq + 1)) & 1u) ? 0xffff0000u : 0u);
    keep1 = (((gmask >> (2 * tq + 8)) & 1u) ? 0x0000ffffu : 0u) |
            (((gmask >> (2 * tq + 9)) & 1u) ? 0xffff0000u : 0u);
  }
  const int vrow = tok + (mi >> 1) * 8 + (lane & 7);
  auto load_v = [&](uint32_t (&va)[D / 16][4]) {
#pragma unroll
    for (int i = 0; i < D / 16; ++i) {
      const int d = i * 16 + (mi & 1) * 8;
      const int c = d / S::kChunkElems;
      const int dc = d - c * S::kChunkElems;
      ldsm_x4_t(vbase + c * S::kRegionBytes + swizzle_offset(vrow * S::kChunkBytes + dc * 2, sw),
                va[i][0], va[i][1], va[i][2], va[i][3]);
      va[i][0] &= keep0;
      va[i][1] &= keep0;
      va[i][2] &= keep1;
      va[i][3] &= keep1;
    }
  };
  uint32_t va[D / 16][4];
  // ---- S^T = K Q^T, two independent accumulation chains over the k-steps ----
  float sa[NT][4], sb[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int e = 0; e < 4; ++e) sa[nt][e] = sb[nt][e] = 0.f;
  const int krow = tok + (mi & 1) * 8 + (lane & 7);
  uint32_t ka[D / 16][4];
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const int d = kk * 16 + (mi >> 1) * 8;
    const int c = d / S::kChunkElems;
    const int dc = d - c * S::kChunkElems;
    ldsm_x4(kbase + c * S::kRegionBytes + swizzle_offset(krow * S::kChunkBytes + dc * 2, sw),
            ka[kk][0], ka[kk][1], ka[kk][2], ka[kk][3]);
  }
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      if (kk & 1)
        mma_16816<E>(sb[nt], ka[kk], qb[nt][kk][0], qb[nt][kk][1]);
      else
        mma_16816<E>(sa[nt], ka[kk], qb[nt][kk][0], qb[nt][kk][1]);
    }
  }
  // ---- mask (keys g, g+8 of this step), scale, online softmax per head ----
  const bool v_lo = (gmask >> g) & 1u;
  const bool v_hi = (gmask >> (g + 8)) & 1u;
  float p[NT][4];
  float alpha[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float s0 = v_lo ? (sa[nt][0] + sb[nt][0]) * scale_log2 : -INFINITY;
    float s1 = v_lo ? (sa[nt][1] + sb[nt][1]) * scale_log2 : -INFINITY;
    float s2 = v_hi ? (sa[nt][2] + sb[nt][2]) * scale_log2 : -INFINITY;
    float s3 = v_hi ? (sa[nt][3] + sb[nt][3]) * scale_log2 : -INFINITY;
    float mx0 = fmaxf(s0, s2);  // head 2t
    float mx1 = fmaxf(s1, s3);  // head 2t+1
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
    }
    const float mn0 = fmaxf(m[nt][0], mx0);
    const float mn1 = fmaxf(m[nt][1], mx1);
    const float base0 = mn0 == -INFINITY ? 0.f : mn0;
    const float base1 = mn1 == -INFINITY ? 0.f : mn1;
    alpha[nt][0] = fast_exp2(m[nt][0] - base0);
    alpha[nt][1] = fast_exp2(m[nt][1] - base1);
    m[nt][0] = mn0;
    m[nt][1] = mn1;
    p[nt][0] = fast_exp2(s0 - base0);
    p[nt][1] = fast_exp2(s1 - base1);
    p[nt][2] = fast_exp2(s2 - base0);
    p[nt][3] = fast_exp2(s3 - base1);
    l[nt][0] = l[nt][0] * alpha[nt][0] + (p[nt][0] + p[nt][2]);
    l[nt][1] = l[nt][1] * alpha[nt][1] + (p[nt][1] + p[nt][3]);
    // Rescale only when some running max of this warp moved.
    if (__any_sync(0xffffffffu, alpha[nt][0] != 1.f || alpha[nt][1] != 1.f)) {
#pragma unroll
      for (int i = 0; i < D / 16; ++i) {
        oT[nt][i][0] *= alpha[nt][0];
        oT[nt][i][1] *= alpha[nt][1];
        oT[nt][i][2] *= alpha[nt][0];
        oT[nt][i][3] *= alpha[nt][1];
      }
    }
  }
  // ---- P^T into B-operand layout (transpose each 8x8 half) ----
  uint32_t pb[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    pb[nt][0] = movmatrix_trans(pack2<E>(p[nt][0], p[nt][1]));  // keys 0-7
    pb[nt][1] = movmatrix_trans(pack2<E>(p[nt][2], p[nt][3]));  // keys 8-15
  }
  // ---- O^T += V^T P^T (V rows of keys that are not real tokens are zeroed:
  // 0 * NaN would leak) ----
  load_v(va);
#pragma unroll
  for (int i = 0; i < D / 16; ++i) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) mma_16816<E>(oT[nt][i], va[i], pb[nt][0], pb[nt][1]);
  }
}

}  // namespace b200
