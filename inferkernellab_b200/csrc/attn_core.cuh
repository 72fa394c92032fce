// Building blocks shared by the paged decode and paged prefill kernels.
//
//   KvTileShape<D>   -- shared-memory geometry of one 64-token K/V tile as TMA
//                       writes it: `chunks` column regions of 64 rows x
//                       chunk_bytes, each 1024-byte aligned, optionally swizzled.
//   issue_kv_tile()  -- producer side: block-table lookup, validity mask,
//                       expect-tx and the TMA loads of one tile (one warp).
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

// Producer (whole warp): load logical tokens tok0 .. tok0+ntok-1 (ntok <= 64) of
// table row `row` and kv head `head` into stage buffers kdst/vdst, arm `bar`,
// and return the token-validity mask (bit i = tile row i holds a real token).
// Pages whose block id is outside [0, num_blocks) are not loaded and masked.
template <int D>
__device__ __forceinline__ void issue_kv_tile(const CUtensorMap* kmap, const CUtensorMap* vmap,
                                              const PagedSource& src, int row, int head, int tok0,
                                              int ntok, uint8_t* kdst, uint8_t* vdst,
                                              uint64_t* bar, uint64_t* mask_out,
                                              uint32_t* err, int lane) {
  using S = KvTileShape<D>;
  const int rows = src.box_rows;
  const int boxes = kKvTile / rows;
  const uint32_t box_bytes = static_cast<uint32_t>(rows) * S::kChunkBytes;
  const long long row_base = static_cast<long long>(row) * src.table_stride;
  uint32_t mlo = 0, mhi = 0, nvalid = 0;
  for (int j0 = 0; j0 < boxes; j0 += 32) {
    const int j = j0 + lane;
    bool ok = false;
    if (j < boxes && j * rows < ntok) {
      const int pos = tok0 + j * rows;
      const long long blk = load_index(src.tables, row_base + pos / src.block_size, src.table64);
      ok = blk >= 0 && blk < src.num_blocks;
      if (!ok && err) atomicOr(err, kErrBadBlock);
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
      const long long blk = load_index(src.tables, row_base + pos / src.block_size, src.table64);
      if (blk >= 0 && blk < src.num_blocks) {
        const int z = static_cast<int>(src.layer_slot_base + blk * src.block_size +
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

// One 16-key step of attention for a 16-row block held by one warp.
//   kbase/vbase: shared addresses of the stage's K/V tile; `tok` = first tile
//   row of the 16 keys; gmask = validity of those 16 keys (bit i = key tok+i).
//   CAUSAL: additionally key (key_pos0 + i) must be < lim0 (row g) / lim1 (row g+8).
template <typename E, int D, bool CAUSAL>
__device__ __forceinline__ void attend16(const uint32_t (&qf)[D / 16][4], float (&o)[D / 8][4],
                                         float (&m_r)[2], float (&l_r)[2], uint32_t kbase,
                                         uint32_t vbase, int tok, uint32_t gmask, int key_pos0,
                                         int lim0, int lim1, float scale_log2, uint32_t sw,
                                         int lane) {
  using S = KvTileShape<D>;
  const int tq = lane & 3;
  float sacc[2][4];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt) {
    sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
    const int trow = tok + nt * 8 + (lane & 7);
    if constexpr (D == 16) {
      const int d = ((lane >> 3) & 1) * 8;
      const uint32_t addr = kbase + swizzle_offset(trow * S::kChunkBytes + d * 2, sw);
      uint32_t b0, b1;
      ldsm_x2(addr, b0, b1);
      mma_16816<E>(sacc[nt], qf[0], b0, b1);
    } else {
#pragma unroll
      for (int kk = 0; kk < D / 16; kk += 2) {
        const int d = kk * 16 + (lane >> 3) * 8;
        const int c = d / S::kChunkElems;
        const int dc = d - c * S::kChunkElems;
        const uint32_t addr =
            kbase + c * S::kRegionBytes + swizzle_offset(trow * S::kChunkBytes + dc * 2, sw);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(addr, b0, b1, b2, b3);
        mma_16816<E>(sacc[nt], qf[kk], b0, b1);
        mma_16816<E>(sacc[nt], qf[kk + 1], b2, b3);
      }
    }
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
  // V rows of keys that are not real tokens are zeroed so NaN/Inf in unwritten
  // slots cannot leak (0 * NaN = NaN).  Causally masked keys are real tokens
  // with finite values by contract and only need P = 0.
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
    const uint32_t addr =
        vbase + c * S::kRegionBytes + swizzle_offset(vrow * S::kChunkBytes + dc * 2, sw);
    uint32_t b0, b1, b2, b3;
    ldsm_x4_t(addr, b0, b1, b2, b3);
    b0 &= keep0;
    b2 &= keep0;
    b1 &= keep1;
    b3 &= keep1;
    mma_16816<E>(o[dt], pa, b0, b1);
    mma_16816<E>(o[dt + 1], pa, b2, b3);
  }
}

}  // namespace b200
