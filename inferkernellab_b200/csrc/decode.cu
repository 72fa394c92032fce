// Paged decode attention for sm_100a: split-KV over a persistent stream-K grid.
//
// Work decomposition
//   A *segment* is one (request r, group of HB kv heads) pair; it owns
//   ceil(len_r / T) *tiles* of T = 64 / HB logical tokens x HB heads (64 K and
//   64 V rows either way).  HB = 1 unless head-group tiles apply (below).  All
//   segments are laid end to end (request major, then head group) and the
//   resulting tile range is cut into equal contiguous pieces, one per CTA
//   ("stream-K"): gridDim.x of them, or fewer on small problems, where the
//   piece length follows the longest segment so that a long request is not
//   split into more pieces than its merge can absorb; short segments that all
//   fit the grid run unsplit, one CTA each.  A CTA therefore walks whole
//   segments plus at most one partial segment at each end, and every CTA moves
//   the same number of K/V bytes whatever the context-length spread.
//   A segment covered by one CTA is written straight to `out`; a segment split
//   over several CTAs writes a partial (normalised O and log-sum-exp) into the
//   workspace, and the CTA that arrives last on the segment's counter merges the
//   partials in one pass (lse and O of several pieces per batch of loads) and
//   resets the counter -- no second kernel, no spin waiting.
//
// Head-group tiles (HB = 2 or 4; head_dim 64/128, G * HB <= 16, T <= block
// size): a tile is one TMA box per tensor -- T tokens of HB heads out of one
// page, through the 4-D head-group tensor map -- instead of one box per page
// and 128-byte chunk of a single head.  TMA moves bytes at a rate set largely
// by the number of boxes; at Hkv = 8, D = 128, block size 16 a tile is two
// 16 KB boxes instead of sixteen 2 KB ones (a pure streaming probe of the
// config-3 cache: 6.94 TB/s against 6.34).  The boxes land head-major, so
// consumer warp w still reads tile rows 16w .. 16w+15.
//
// Inside a CTA
//   warp 4 (producer): reads the block table for each tile and issues TMA tile
//     loads of the K and V page rows of the segment's heads into a
//     STAGES-deep shared-memory ring (mbarrier full/empty pipeline, bounded
//     waits);
//   warps 0..3 (consumers): the G = Hq/Hkv query heads of the segment form the
//     M dimension of mma.sync m16n8k16 tiles (padded to 16 rows per m-tile);
//     S = Q K^T and O += P V run on the tensor cores with fp32 accumulation and
//     a base-2 online softmax.  Each consumer warp owns 16 rows of every tile
//     (a token slice of one head); the slices of a head are merged through
//     shared memory at segment end.
//
// Masking (reference triton_ops.py:128-165): tokens at or past the context
// length, and tokens of pages whose block id is outside [0, num_blocks), get
// score -inf and their V rows are zeroed in registers, so NaN/Inf left in
// unwritten cache slots never reaches the output.
#include <math.h>

#include <mutex>

#include "../../include/b200_paged_attn.h"
#include "attn_core.cuh"
#include "common.cuh"
#include "decode.h"
#include "host_common.h"

namespace b200 {

constexpr int kDecTile = kKvTile;
constexpr int kDecConsumerWarps = 4;
constexpr int kDecThreads = (kDecConsumerWarps + 1) * 32;
constexpr int kDecMaxSeqs = 8192;

struct DecodeParams {
  const void* q;
  void* out;
  const void* tables;
  const void* lens;
  uint32_t* err;
  int* counters;
  float* part_lse;
  float* part_o;
  long long q_stride_seq, q_stride_head;
  long long out_stride_seq, out_stride_head;
  long long table_stride;
  long long layer_slot_base;
  int num_seqs, num_kv_heads, group, table_width;
  int num_blocks, block_size;
  int box_rows, sw_mask;
  int heads_per_tile;  // HB: kv heads per tile (1, 2 or 4)
  int tile_tokens;     // T = 64 / HB tokens per tile
  int table64, lens64;
  float scale_log2;
  // Fused new-token append (b200_paged_decode_append); fuse_append == 0 = off.
  // The new token of request r is its last context position (lens[r] - 1): the
  // CTA that owns the tile holding that position writes its K (rotated when
  // rope) and V at new_slots[r] before its first TMA load; with rope every CTA
  // also stages the rotated q of its segments in `out`.
  int fuse_append, rope, slots64;
  const void* new_k;
  const void* new_v;
  const void* cos;
  const void* sin;
  const void* new_slots;
  void* k_cache;
  void* v_cache;
  long long nk_stride_seq, nk_stride_head, nv_stride_seq, nv_stride_head;
  long long cos_stride, sin_stride;
  long long slots_per_layer;
};

// Ring depth per CTA and CTAs per SM (kDecMinBlocks feeds __launch_bounds__).
constexpr int kDecMinBlocks = 2;
template <int D>
struct DecodeShape : KvTileShape<D> {
  static constexpr int kStages = D >= 128 ? 3 : 4;
};

// Shared-memory carve-up (offsets from a 1024-byte aligned base).
struct DecodeSmem {
  int stage_bytes;  // K + V of one stage
  int bars_off;     // full[S], empty[S]
  int mask_off;     // uint64 per stage
  int flags_off;    // abort, merge flag, most tiles of one segment
  int red_m_off, red_l_off, red_w_off, row_off, red_o_off, merge_w_off;
  int table_off;    // producer's block-table window
  int len_off, begin_off, scan_off;
  int total;
};

constexpr int kMergeChunk = 32;  // split pieces merged per pass

// Rows of one segment's reduction arrays: the transposed variants hold at most
// 16 query heads per segment (G * HB <= 16), the heads-as-M ones 16 * MT.
template <int MT>
constexpr int decode_seg_rows() {
  return MT < 0 ? 16 : 16 * MT;
}

// `group` = G, `hb` = kv heads per tile.  The slice reduction arrays hold
// (slices per head) x (G * hb) rows = kSlices x G whatever hb is.
template <int D, int MT>
__host__ __device__ inline DecodeSmem decode_smem_layout(int group, int hb, int num_seqs) {
  using S = DecodeShape<D>;
  constexpr int kSlices = MT < 0 ? kDecConsumerWarps : kDecConsumerWarps / MT;
  constexpr int kRows = MT < 0 ? 8 * -MT : 16 * MT;
  DecodeSmem L;
  L.stage_bytes = 2 * S::kTileBytes;
  int off = S::kStages * L.stage_bytes;
  L.bars_off = off;
  off += 2 * S::kStages * 8;
  L.mask_off = off;
  off += S::kStages * 8;
  L.flags_off = off;
  off += 16;
  L.red_m_off = off;
  off += kSlices * kRows * 4;
  L.red_l_off = off;
  off += kSlices * kRows * 4;
  L.red_w_off = off;
  off += kSlices * kRows * 4;
  L.row_off = off;  // base and 1/l (or sum) per segment row
  off += 2 * decode_seg_rows<MT>() * 4;
  off = (off + 15) & ~15;
  L.red_o_off = off;
  off += kSlices * group * D * 4;
  L.merge_w_off = off;
  off += kMergeChunk * group * hb * 4;
  L.table_off = off;
  off += kTableWindow * 4;
  L.len_off = off;
  off += num_seqs * 4;
  L.begin_off = off;
  off += (num_seqs + 1) * 4;
  L.scan_off = off;
  off += (kDecThreads / 32) * 4;
  L.total = off;
  return L;
}

// Walks tiles in global order: request-major, then head group h (of
// `groups` = Hkv / HB), then tile t (of nt = ceil(len / tile_tokens)).
struct TileCursor {
  int r, h, t, nt;
  __device__ void init(int tile, const int* begin, const int* lens, int num_seqs,
                       int tile_tokens) {
    int lo = 0, hi = num_seqs;
    while (hi - lo > 1) {
      int mid = (lo + hi) >> 1;
      if (begin[mid] <= tile) lo = mid; else hi = mid;
    }
    r = lo;
    nt = (lens[r] + tile_tokens - 1) / tile_tokens;
    int local = tile - begin[r];
    h = local / nt;
    t = local - h * nt;
  }
  __device__ void advance(const int* lens, int num_seqs, int groups, int tile_tokens) {
    if (++t < nt) return;
    t = 0;
    if (++h < groups) return;
    h = 0;
    do {
      ++r;
    } while (r < num_seqs && lens[r] == 0);
    nt = r < num_seqs ? (lens[r] + tile_tokens - 1) / tile_tokens : 0;
  }
};

// The consumer warps, while the producer already streams the first tiles:
//  * write the new token (position len - 1) of every segment whose last tile
//    lies in [my_begin, my_end) -- only this CTA loads that tile, so no other CTA
//    can read the token's cache row.  K is rotated with the reference's rounding
//    when p.rope, V is copied;
//  * with p.rope, rotate the query heads of every segment the range touches and
//    stage them in the segment's own rows of `out` (the consumers read q from
//    there).  A segment's output is written only after every CTA working on it
//    has passed this prologue, and CTAs sharing a split segment write identical
//    bits here.
// 16-byte vectors (the host checks the alignment); every item issues its data
// loads before the slot load, so it costs one memory round trip.
template <typename E>
__device__ __forceinline__ void rope_vec8(const uint4& a4, const uint4& b4, const uint4& cl4,
                                          const uint4& ch4, const uint4& sl4, const uint4& sh4,
                                          uint4& lo4, uint4& hi4) {
  using T = typename E::T;
  const T* a = reinterpret_cast<const T*>(&a4);
  const T* b = reinterpret_cast<const T*>(&b4);
  const T* cl = reinterpret_cast<const T*>(&cl4);
  const T* ch = reinterpret_cast<const T*>(&ch4);
  const T* sl = reinterpret_cast<const T*>(&sl4);
  const T* sh = reinterpret_cast<const T*>(&sh4);
  T* lo = reinterpret_cast<T*>(&lo4);
  T* hi = reinterpret_cast<T*>(&hi4);
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    float l, u;
    rope_pair<E>(to_float<E>(a[e]), to_float<E>(b[e]), to_float<E>(cl[e]), to_float<E>(sl[e]),
                 to_float<E>(ch[e]), to_float<E>(sh[e]), l, u);
    lo[e] = from_float<E>(l);
    hi[e] = from_float<E>(u);
  }
}

template <typename E, int D>
__device__ __forceinline__ void fused_prologue(const DecodeParams& p, const int* begin_s,
                                               const int* len_s, int my_begin, int my_end,
                                               int thread, int nthreads) {
  using T = typename E::T;
  constexpr int kVec = D / 8;    // 16-byte vectors per row
  constexpr int kHalf = kVec / 2;
  constexpr int kUnroll = 4;     // items per thread whose loads are in flight together
  const int hkv = p.num_kv_heads;
  const int kv_items = 2 * kVec;                       // V vectors, then K vectors / pairs
  const int q_items = p.rope ? p.group * kHalf : 0;    // rotary pairs of the G query heads
  const int per_seg = kv_items + q_items;
  // Segments are (request, head group); an item belongs to one kv head of the
  // segments this range touches: kv-head unit u = r * hkv + h, and segment g
  // covers units g * hb .. g * hb + hb - 1.
  const int hb = p.heads_per_tile;
  const int groups = hkv / hb;
  TileCursor first, last;
  first.init(my_begin, begin_s, len_s, p.num_seqs, p.tile_tokens);
  last.init(my_end - 1, begin_s, len_s, p.num_seqs, p.tile_tokens);
  const int g0 = first.r * groups + first.h;
  const int total = (last.r * groups + last.h - g0 + 1) * hb * per_seg;
  enum : int { kNone = 0, kV = 1, kK = 2, kQ = 3 };
  for (int base = thread; base < total; base += nthreads * kUnroll) {
    int kind[kUnroll], r_[kUnroll], h_[kUnroll], j_[kUnroll];
    long long slot[kUnroll], head_[kUnroll];
    uint4 x0[kUnroll], x1[kUnroll], c0[kUnroll], c1[kUnroll], s0[kUnroll], s1[kUnroll];
    // Phase 1: decode every item and issue all of its loads.
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      kind[u] = kNone;
      const int it = base + u * nthreads;
      if (it >= total) continue;
      const int k = it / per_seg;
      const int item = it - k * per_seg;
      const int unit = g0 * hb + k;
      const int r = unit / hkv;
      const int h = unit - r * hkv;
      const int len = len_s[r];
      if (len == 0) continue;
      r_[u] = r;
      h_[u] = h;
      const bool rope = p.rope != 0;
      if (item >= kv_items) {
        const int qi = item - kv_items;
        const int qh = qi / kHalf;
        const int j = qi - qh * kHalf;
        const long long head = static_cast<long long>(h) * p.group + qh;
        const uint4* qs = reinterpret_cast<const uint4*>(
            reinterpret_cast<const T*>(p.q) + r * p.q_stride_seq + head * p.q_stride_head);
        x0[u] = qs[j];
        x1[u] = qs[j + kHalf];
        j_[u] = j;
        head_[u] = head;
        kind[u] = kQ;
      } else {
        const int nt = (len + p.tile_tokens - 1) / p.tile_tokens;
        const int last_tile = begin_s[r] + (h / hb) * nt + nt - 1;
        if (last_tile < my_begin || last_tile >= my_end) continue;
        if (item < kVec) {
          x0[u] = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.new_v) +
                                                 r * p.nv_stride_seq + h * p.nv_stride_head)[item];
          j_[u] = item;
          kind[u] = kV;
        } else {
          const int j = item - kVec;
          if (rope && j >= kHalf) continue;  // the pair (j, j + D/16) is handled by item j
          const uint4* ks = reinterpret_cast<const uint4*>(
              reinterpret_cast<const T*>(p.new_k) + r * p.nk_stride_seq + h * p.nk_stride_head);
          x0[u] = ks[j];
          if (rope) x1[u] = ks[j + kHalf];
          j_[u] = j;
          kind[u] = kK;
        }
        slot[u] = load_index(p.new_slots, r, p.slots64);
      }
      if (rope && kind[u] != kV) {
        const uint4* cv = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.cos) +
                                                         r * p.cos_stride);
        const uint4* sv = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.sin) +
                                                         r * p.sin_stride);
        const int j = j_[u];
        c0[u] = cv[j];
        c1[u] = cv[j + kHalf];
        s0[u] = sv[j];
        s1[u] = sv[j + kHalf];
      }
    }
    // Phase 2: rotate and store.
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      if (kind[u] == kNone) continue;
      const int r = r_[u], h = h_[u], j = j_[u];
      if (kind[u] == kQ) {
        uint4 lo, hi;
        rope_vec8<E>(x0[u], x1[u], c0[u], c1[u], s0[u], s1[u], lo, hi);
        uint4* qd = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + r * p.out_stride_seq +
                                             head_[u] * p.out_stride_head);
        qd[j] = lo;
        qd[j + kHalf] = hi;
        continue;
      }
      if (slot[u] < 0) continue;  // padding slot: nothing to append
      if (slot[u] >= p.slots_per_layer) {
        if (kind[u] == kV && j == 0 && p.err) atomicOr(p.err, kErrBadSlot);
        continue;
      }
      const long long row = ((p.layer_slot_base + slot[u]) * hkv + h) * D;
      if (kind[u] == kV) {
        reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.v_cache) + row)[j] = x0[u];
        continue;
      }
      uint4* kd = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.k_cache) + row);
      if (p.rope) {
        uint4 lo, hi;
        rope_vec8<E>(x0[u], x1[u], c0[u], c1[u], s0[u], s1[u], lo, hi);
        kd[j] = lo;
        kd[j + kHalf] = hi;
      } else {
        kd[j] = x0[u];
      }
    }
  }
}

__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Store four consecutive output elements (8 bytes).
template <typename E>
__device__ __forceinline__ void store4(typename E::T* dst, float4 v) {
  uint2 packed;
  packed.x = pack2<E>(v.x, v.y);
  packed.y = pack2<E>(v.z, v.w);
  *reinterpret_cast<uint2*>(dst) = packed;
}

constexpr int kMinTilesPerCta = 2;  // fewer split pieces on small problems
// Problems with fewer tiles than this per CTA of the grid size their ranges to
// the longest segment (see the range choice); bigger ones are cut into
// grid-many equal ranges.
constexpr int kAdaptMaxTiles = 32;
// A segment of at most this many tiles is not split when the grid has a CTA
// for every segment (see the range choice).
constexpr int kSegWholeMaxTiles = 10;

// A CTA for every segment, and few enough tiles that no segment can be longer
// than the limit on average (config-3-sized batches skip the length pass).
__device__ __forceinline__ bool decode_whole_segs_possible(int segments, int tiles, int grid) {
  return segments <= grid && tiles <= segments * kSegWholeMaxTiles;
}

// FUSED: the new-token append (and rotary embedding) of b200_paged_decode_append
// is compiled in; the plain decode instantiation carries none of that code.
template <typename E, int D, int MT, bool FUSED>
__global__ void __launch_bounds__(kDecThreads, kDecMinBlocks)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const DecodeParams p) {
  using S = DecodeShape<D>;
  using T = typename E::T;
  // MT > 0: query heads are the MMA M rows (MT m-tiles of 16, for G > 16).
  // MT < 0: transposed form, keys are M and the group is N = 8 * (-MT) (G <= 16).
  constexpr bool kTrans = MT < 0;
  constexpr int NT = kTrans ? -MT : 1;
  constexpr int kSlices = kTrans ? kDecConsumerWarps : kDecConsumerWarps / MT;
  constexpr int kRows = kTrans ? 8 * NT : 16 * MT;
  constexpr int kTokPerWarp = kDecTile / kSlices;  // 16, 32 or 64
  constexpr int kGroups16 = kTokPerWarp / 16;
  constexpr int kStages = S::kStages;
  constexpr int kConsumers = kDecConsumerWarps * 32;
  constexpr int kD4 = D / 4;
  constexpr int kElems4 =
      (decode_seg_rows<MT>() * kD4 + kConsumers - 1) / kConsumers;  // float4 per thread

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const DecodeSmem L = decode_smem_layout<D, MT>(p.group, p.heads_per_tile, p.num_seqs);
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + L.bars_off);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* stage_mask = reinterpret_cast<uint64_t*>(smem + L.mask_off);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L.flags_off);
  int* merge_flag = reinterpret_cast<int*>(smem + L.flags_off + 4);
  int* max_seg_tiles = reinterpret_cast<int*>(smem + L.flags_off + 8);
  float* red_m = reinterpret_cast<float*>(smem + L.red_m_off);
  float* red_l = reinterpret_cast<float*>(smem + L.red_l_off);
  float* red_w = reinterpret_cast<float*>(smem + L.red_w_off);
  float* row_base = reinterpret_cast<float*>(smem + L.row_off);
  float* row_l = row_base + decode_seg_rows<MT>();
  float* red_o = reinterpret_cast<float*>(smem + L.red_o_off);
  float* merge_w = reinterpret_cast<float*>(smem + L.merge_w_off);
  int* len_s = reinterpret_cast<int*>(smem + L.len_off);
  int* begin_s = reinterpret_cast<int*>(smem + L.begin_off);
  int* scan_s = reinterpret_cast<int*>(smem + L.scan_off);

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int B = p.num_seqs;
  const int HKV = p.num_kv_heads;
  const int G = p.group;
  const int HB = p.heads_per_tile;  // kv heads per tile
  const int HG = HKV / HB;          // head groups (segments per request)
  const int TT = p.tile_tokens;     // tokens per tile
  const int GH = G * HB;            // query heads per segment

  // ---- prologue: effective lengths and the tile prefix over requests ----
  // Launched with programmatic stream serialization, this grid may start while
  // the previous kernel on the stream is finishing: only barrier set-up and the
  // tensor-map prefetch (kernel parameters) run before griddepcontrol.wait,
  // which returns once that kernel has completed and its writes are visible.
  // Every global access comes after it.
  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kDecConsumerWarps);
    }
    *abort_flag = 0;
    *max_seg_tiles = 0;
    fence_mbar_init();
  }
  if (warp == kDecConsumerWarps && lane == 0) {
    tma_prefetch_desc(&kmap);
    tma_prefetch_desc(&vmap);
  }
  // While the previous kernel may still run: L2 prefetch of the metadata that
  // the prologue and the producer read first -- the lengths (CTA c takes lines
  // c, c + grid, ...) and the block-table rows (CTA c takes rows c, c + grid,
  // ...).  Between the layers of a model the weight stream evicts them from L2;
  // this turns the first two dependent loads after the wait into L2 hits.
  if (warp < kDecConsumerWarps) {
    const int cw = kDecConsumerWarps * 32;
    const long long lens_bytes = static_cast<long long>(B) * (p.lens64 ? 8 : 4);
    const long long lens_lines = (lens_bytes + 127) / 128 + 1;  // base need not be aligned
    for (long long ln = blockIdx.x; ln < lens_lines; ln += gridDim.x) {
      const long long lo = ln * 128 - (reinterpret_cast<uintptr_t>(p.lens) & 127);
      const long long s0 = lo < 0 ? 0 : lo;
      const long long s1 = lo + 128 < lens_bytes ? lo + 128 : lens_bytes;
      if (s1 > s0) prefetch_l2_span(static_cast<const char*>(p.lens) + s0, s1 - s0, tid, cw);
    }
    // Only a table of at most 4 MiB: a table whose rows are far wider than the
    // contexts (capacity for very long requests) would otherwise pull mostly
    // unread bytes from DRAM.
    const int esz = p.table64 ? 8 : 4;
    if (static_cast<long long>(B) * p.table_width * esz <= (4ll << 20))
      for (int r = blockIdx.x; r < B; r += gridDim.x)
        prefetch_l2_span(static_cast<const char*>(p.tables) + static_cast<long long>(r) * p.table_stride * esz,
                         static_cast<long long>(p.table_width) * esz, tid, cw);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The next kernel on the stream may be scheduled now; its CTAs run their own
  // set-up on SMs this grid leaves and then wait for it to complete.
  if (tid == 0) asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  const long long cap = static_cast<long long>(p.table_width) * p.block_size;
  for (int i = tid; i < B; i += kDecThreads) {
    long long len = load_index(p.lens, i, p.lens64);
    len = len < 0 ? 0 : (len > cap ? cap : len);
    len_s[i] = static_cast<int>(len);
  }
  __syncthreads();
  {
    const int chunk = (B + kDecThreads - 1) / kDecThreads;
    const int lo = min(B, tid * chunk);
    const int hi = min(B, lo + chunk);
    int sum = 0;
    for (int i = lo; i < hi; ++i) sum += ((len_s[i] + TT - 1) / TT) * HG;
    int total_all = 0;
    int acc = block_exclusive_scan<kDecThreads>(sum, scan_s, &total_all);
    for (int i = lo; i < hi; ++i) {
      begin_s[i] = acc;
      acc += ((len_s[i] + TT - 1) / TT) * HG;
    }
    if (tid == 0) begin_s[B] = total_all;
    // The longest segment, only where whole segments are possible at all or
    // the problem is small enough for the split size to depend on it.
    if (decode_whole_segs_possible(B * HG, total_all, static_cast<int>(gridDim.x)) ||
        total_all < static_cast<int>(gridDim.x) * kAdaptMaxTiles) {
      int most = 0;
      for (int i = lo; i < hi; ++i) most = max(most, (len_s[i] + TT - 1) / TT);
      if (most > 0) atomicMax(max_seg_tiles, most);
    }
  }
  __syncthreads();

  // Requests with no readable token: NaN, like 0/0 in the reference kernel.
  // Each consumer thread of CTA 0 checks its share of the requests (this CTA
  // must not spend a serial pass over the batch before it starts streaming).
  if (blockIdx.x == 0 && warp < kDecConsumerWarps) {
    for (int r = tid; r < B; r += kConsumers) {
      if (len_s[r] != 0) continue;
      const int nh = HKV * G;
      for (int i = 0; i < nh * D; ++i) {
        const int hq = i / D, d = i - hq * D;
        reinterpret_cast<T*>(p.out)[r * p.out_stride_seq + hq * p.out_stride_head + d] =
            from_float<E>(__int_as_float(0x7fc00000));
      }
    }
  }

  // ---- this CTA's contiguous range of tiles (stream-K) ----
  // On small batches a split piece (publish + merge of the pieces) costs
  // several us against ~1 us per tile (~8 us in the heads-as-M variants), so
  // when every segment is short and the grid has a CTA for each, CTA b takes
  // segment b whole and nothing is split.  Otherwise the tiles are cut into
  // equal ranges.
  const int total = begin_s[B];
  const bool whole_segs = decode_whole_segs_possible(B * HG, total, static_cast<int>(gridDim.x)) &&
                          *max_seg_tiles <= kSegWholeMaxTiles;
  // Split size t (tiles per range).  A segment of n tiles cut into ranges of t
  // is merged from ~n / t pieces, ~n / (t * kMergePB) dependent L2 round trips
  // for the CTA that merges, against t tiles of streaming in every CTA; t ~
  // sqrt(n * 1.4 / kMergePB) balances the two (1.4 ~ a loaded L2 round trip
  // over one tile's streaming time, measured on B200: single long requests
  // ran up to 40 % faster than with t = 2, configs 1-5 are unchanged).
  constexpr int kMergePB = kTrans ? 16 / kElems4 : 4;  // pieces per merge round trip
  int min_tiles = kMinTilesPerCta;
  if (total < static_cast<int>(gridDim.x) * kAdaptMaxTiles) {
    float t = sqrtf(static_cast<float>(*max_seg_tiles) * (1.4f / kMergePB));
    // Heads-as-M: the nearest power of two, which divides the power-of-two
    // segment lengths of uniform batches (t = 3 on 32-tile segments left more
    // CTAs straddling two segments, each with two pieces to publish).
    if constexpr (!kTrans) t = exp2f(rintf(log2f(fmaxf(t, 1.f))));
    min_tiles = max(min_tiles, static_cast<int>(t));
  }
  const int ctas = whole_segs ? B * HG
                              : min(static_cast<int>(gridDim.x),
                                    max(1, (total + min_tiles - 1) / min_tiles));
  if (static_cast<int>(blockIdx.x) >= ctas) return;
  int per_cta, my_begin, my_end;
  if (whole_segs) {
    const int r = static_cast<int>(blockIdx.x) / HG;
    const int h = static_cast<int>(blockIdx.x) - r * HG;
    const int nt = (len_s[r] + TT - 1) / TT;
    my_begin = begin_s[r] + h * nt;
    my_end = my_begin + nt;
    per_cta = max(1, nt);  // every segment is complete: no piece slots are used
  } else {
    per_cta = (total + ctas - 1) / ctas;
    my_begin = min(total, static_cast<int>(blockIdx.x) * per_cta);
    my_end = min(total, my_begin + per_cta);
  }
  const int n_tiles = my_end - my_begin;
  if (n_tiles <= 0) return;
  // Fused append: the consumers write the new tokens (and stage the rotated q)
  // while the producer streams; the producer waits on named barrier 2 only
  // before the first tile that holds a new token.
  constexpr uint32_t kBarAppended = 2;
  if constexpr (FUSED) {
    if (warp < kDecConsumerWarps) {
      fused_prologue<E, D>(p, begin_s, len_s, my_begin, my_end, tid, kDecConsumerWarps * 32);
      // Generic-proxy cache writes -> visible to the producer's TMA loads.
      asm volatile("fence.proxy.async.global;" ::: "memory");
      named_bar_arrive(kBarAppended, kDecThreads);
      named_bar_sync(1, kDecConsumerWarps * 32);  // staged q visible to every consumer
    }
  }

  const uint32_t smem_base = smem_u32(smem);

  if (warp == kDecConsumerWarps) {
    // =============================== producer ===============================
    PagedSource src;
    src.tables = p.tables;
    src.table_stride = p.table_stride;
    src.layer_slot_base = p.layer_slot_base;
    src.table64 = p.table64;
    src.num_blocks = p.num_blocks;
    src.block_size = p.block_size;
    src.box_rows = p.box_rows;
    TableWindow win;
    win.ids = reinterpret_cast<int*>(smem + L.table_off);
    win.row = -1;
    win.first = 0;
    win.count = 0;
    TileCursor cur;
    cur.init(my_begin, begin_s, len_s, B, TT);
    int issued = 0;
    bool appended = !FUSED;
    for (int it = 0; it < n_tiles; ++it) {
      if (FUSED && !appended && cur.t == cur.nt - 1) {
        named_bar_sync(kBarAppended, kDecThreads);  // the consumers wrote the new tokens
        appended = true;
      }
      const int s = it % kStages;
      const uint32_t k = static_cast<uint32_t>(it / kStages);
      if (!mbar_wait_bounded(&empty_bar[s], (k & 1u) ^ 1u, abort_flag, p.err, kErrWaitEmpty))
        break;
      const int len = len_s[cur.r];
      const int tok0 = cur.t * TT;
      const int ntok = min(TT, len - tok0);
      uint8_t* kdst = smem + s * L.stage_bytes;
      const int row_pages = (len + p.block_size - 1) / p.block_size;
      if (HB > 1)
        issue_kv_tile_heads<true>(&kmap, &vmap, src, win, cur.r, row_pages, cur.h * HB, HB, tok0, ntok,
                            S::kTileBytes, kdst, kdst + S::kTileBytes, &full_bar[s],
                            &stage_mask[s], p.err, lane);
      else
        issue_kv_tile<D, true>(&kmap, &vmap, src, win, cur.r, row_pages, cur.h, tok0, ntok, kdst,
                         kdst + S::kTileBytes, &full_bar[s], &stage_mask[s], p.err, lane);
      ++issued;
      cur.advance(len_s, B, HG, TT);
    }
    if (FUSED && !appended) named_bar_sync(kBarAppended, kDecThreads);
    // Drain: the last phases this warp armed must complete before the CTA
    // exits (bounded; only waits after an abort left stages unconsumed).
    if (lane == 0) drain_stages<kStages>(full_bar, issued, p.err);
    return;
  }

  // ================================ consumers ================================
  const int mt = kTrans ? 0 : warp % (kTrans ? 1 : MT);
  const int slice = kTrans ? warp : warp / (kTrans ? 1 : MT);
  const int g = lane >> 2;
  const int tq = lane & 3;
  const int row0 = mt * 16 + g;  // heads-as-M: query-head row inside the group
  const int row1 = row0 + 8;
  const uint32_t sw = static_cast<uint32_t>(p.sw_mask);
  // Transposed variants: warp w reads tile rows 16w..16w+15, i.e. head hl =
  // w / SPH of the tile's HB heads, token slice w % SPH (SPH = 4 / HB slices per
  // head).  Heads-as-M variants: HB = 1, kSlices slices of MT warps each.
  const int SPH = kTrans ? kDecConsumerWarps / HB : kSlices;
  const int hl = kTrans ? warp / SPH : 0;
  const int sl_h = kTrans ? warp - hl * SPH : slice;  // slice within the head
  const int rstride = kTrans ? GH : kRows;            // reduction-array row stride

  // heads-as-M state
  uint32_t qf[D / 16][4];
  float o[D / 8][4];
  float m_r[2], l_r[2];
  // transposed state
  uint32_t qb[NT][D / 16][2];
  float oT[NT][D / 16][4];
  float m_t[NT][2], l_t[NT][2];
  // Running softmax state to its empty value.  Done at the start and again as
  // soon as a segment's state has been handed to shared memory, so that it holds
  // constants (no live registers) through the publish and merge that follow.
  auto reset_state = [&]() {
    if constexpr (kTrans) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
        for (int i = 0; i < D / 16; ++i) oT[nt][i][0] = oT[nt][i][1] = oT[nt][i][2] = oT[nt][i][3] = 0.f;
        m_t[nt][0] = m_t[nt][1] = -INFINITY;
        l_t[nt][0] = l_t[nt][1] = 0.f;
      }
    } else {
#pragma unroll
      for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
      m_r[0] = m_r[1] = -INFINITY;
      l_r[0] = l_r[1] = 0.f;
    }
  };
  reset_state();
  bool aborted = false;

  TileCursor cur;
  cur.init(my_begin, begin_s, len_s, B, TT);
  bool seg_start = true;

  for (int it = 0; it < n_tiles; ++it) {
    if (seg_start) {
      seg_start = false;
      // With the fused rotary append, the prologue staged the rotated q in `out`.
      const bool staged = FUSED && p.rope;
      const long long qhead0 = static_cast<long long>(cur.h * HB + hl) * G;
      const T* qg = staged ? reinterpret_cast<const T*>(p.out) + cur.r * p.out_stride_seq +
                                 qhead0 * p.out_stride_head
                           : reinterpret_cast<const T*>(p.q) + cur.r * p.q_stride_seq +
                                 qhead0 * p.q_stride_head;
      const long long q_head_stride = staged ? p.out_stride_head : p.q_stride_head;
      if constexpr (kTrans) {
        load_qT_frag<E, D, NT>(qb, qg, q_head_stride, G, lane);
      } else {
        load_q_frag<E, D>(qf, row0 < G ? qg + row0 * q_head_stride : nullptr,
                          row1 < G ? qg + row1 * q_head_stride : nullptr, tq);
      }
    }

    const int s = it % kStages;
    const uint32_t k = static_cast<uint32_t>(it / kStages);
    if (!aborted && !mbar_wait_bounded(&full_bar[s], k & 1u, abort_flag, p.err, kErrWaitFull))
      aborted = true;

    if (!aborted) {
      const uint64_t tmask = stage_mask[s];
      const uint32_t kbase = smem_base + s * L.stage_bytes;
      const uint32_t vbase = kbase + S::kTileBytes;
      if constexpr (kTrans) {
        const int tok = slice * kTokPerWarp;  // one 16-key group per warp
        const uint32_t gmask = static_cast<uint32_t>(tmask >> tok) & 0xffffu;
        if (gmask != 0)
          decode_step16_T<E, D, NT>(qb, oT, m_t, l_t, kbase, vbase, tok, gmask, p.scale_log2, sw,
                                    lane);
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
      } else {
#pragma unroll
        for (int gi = 0; gi < kGroups16; ++gi) {
          const int tok = slice * kTokPerWarp + gi * 16;  // first tile row of this 16-key group
          const uint32_t gmask = static_cast<uint32_t>(tmask >> tok) & 0xffffu;
          if (gmask == 0) continue;
          attend16<E, D, false>(qf, o, m_r, l_r, kbase, vbase, tok, gmask, 0, 0, 0,
                                p.scale_log2, sw, lane);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty_bar[s]);
      }
    }

    // ---- segment end: merge the token slices, then finish or publish ----
    const bool seg_end = (cur.t == cur.nt - 1) || (it == n_tiles - 1);
    if (seg_end) {
      const int seg = cur.r * HG + cur.h;
      const int seg_begin = begin_s[cur.r] + cur.h * cur.nt;
      const int seg_end_tile = seg_begin + cur.nt;
      const bool complete = seg_begin >= my_begin && seg_end_tile <= my_end;
      const int slot = seg_begin <= my_begin ? 2 * blockIdx.x : 2 * blockIdx.x + 1;
      T* out_seg = reinterpret_cast<T*>(p.out) + cur.r * p.out_stride_seq +
                   static_cast<long long>(cur.h * GH) * p.out_stride_head;
      if constexpr (kTrans) {
        // l: reduce each head's partial over the 8 key lanes (g).
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            float v = l_t[nt][j];
            v += __shfl_xor_sync(0xffffffffu, v, 4);
            v += __shfl_xor_sync(0xffffffffu, v, 8);
            v += __shfl_xor_sync(0xffffffffu, v, 16);
            l_t[nt][j] = v;
          }
        if (!aborted) {
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const int h0 = nt * 8 + 2 * tq;
            const int sr = hl * G + h0;  // segment row of query head h0 of this warp's kv head
            if (g == 0) {
              if (h0 < G) {
                red_m[sl_h * rstride + sr] = m_t[nt][0];
                red_l[sl_h * rstride + sr] = l_t[nt][0];
              }
              if (h0 + 1 < G) {
                red_m[sl_h * rstride + sr + 1] = m_t[nt][1];
                red_l[sl_h * rstride + sr + 1] = l_t[nt][1];
              }
            }
#pragma unroll
            for (int i = 0; i < D / 16; ++i) {
              const int d0 = i * 16 + g;
              if (h0 < G) {
                float* dst = red_o + (sl_h * GH + sr) * D;
                dst[d0] = oT[nt][i][0];
                dst[d0 + 8] = oT[nt][i][2];
              }
              if (h0 + 1 < G) {
                float* dst = red_o + (sl_h * GH + sr + 1) * D;
                dst[d0] = oT[nt][i][1];
                dst[d0 + 8] = oT[nt][i][3];
              }
            }
          }
        }
      } else {
        const float l0 = quad_sum(l_r[0]);
        const float l1 = quad_sum(l_r[1]);
        if (!aborted) {
          if (tq == 0) {
            red_m[slice * kRows + row0] = m_r[0];
            red_m[slice * kRows + row1] = m_r[1];
            red_l[slice * kRows + row0] = l0;
            red_l[slice * kRows + row1] = l1;
          }
          if (row0 < G) {
            float* dst = red_o + (slice * G + row0) * D + 2 * tq;
#pragma unroll
            for (int i = 0; i < D / 8; ++i)
              *reinterpret_cast<float2*>(dst + i * 8) = make_float2(o[i][0], o[i][1]);
          }
          if (row1 < G) {
            float* dst = red_o + (slice * G + row1) * D + 2 * tq;
#pragma unroll
            for (int i = 0; i < D / 8; ++i)
              *reinterpret_cast<float2*>(dst + i * 8) = make_float2(o[i][2], o[i][3]);
          }
        }
      }
      reset_state();
      named_bar_sync(1, kConsumers);
      // Per-row slice weights, once per row (segment rows = the GH query heads).
      if (!aborted) {
        for (int row = tid; row < GH; row += kConsumers) {
          float mmax = -INFINITY;
          for (int sl = 0; sl < SPH; ++sl) mmax = fmaxf(mmax, red_m[sl * rstride + row]);
          const float base = mmax == -INFINITY ? 0.f : mmax;
          float lsum = 0.f;
          for (int sl = 0; sl < SPH; ++sl) {
            const float w = fast_exp2(red_m[sl * rstride + row] - base);
            red_w[sl * rstride + row] = w;
            lsum += red_l[sl * rstride + row] * w;
          }
          row_base[row] = base;
          row_l[row] = lsum;
          if (!complete)
            p.part_lse[slot * GH + row] = lsum > 0.f ? base + fast_log2(lsum) : -INFINITY;
        }
      }
      named_bar_sync(1, kConsumers);
      if (!aborted) {
        for (int e = tid; e < GH * kD4; e += kConsumers) {
          const int row = e / kD4;
          const int d4 = e - row * kD4;
          float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
          for (int sl = 0; sl < SPH; ++sl) {
            const float w = red_w[sl * rstride + row];
            const float4 v = reinterpret_cast<const float4*>(red_o + (sl * GH + row) * D)[d4];
            acc.x += w * v.x;
            acc.y += w * v.y;
            acc.z += w * v.z;
            acc.w += w * v.w;
          }
          const float inv = 1.f / row_l[row];
          acc.x *= inv;
          acc.y *= inv;
          acc.z *= inv;
          acc.w *= inv;
          if (complete)
            store4<E>(out_seg + row * p.out_stride_head + d4 * 4, acc);
          else
            reinterpret_cast<float4*>(p.part_o)[(static_cast<long long>(slot) * GH + row) * kD4 +
                                                d4] = acc;
        }
      }
      if (!complete) {
        named_bar_sync(1, kConsumers);
        const int p_first = seg_begin / per_cta;
        const int npieces = (seg_end_tile - 1) / per_cta - p_first + 1;
        if (tid == 0) {
          int last = 0;
          if (!aborted) {
            // One acquire-release RMW: it releases this CTA's piece (the barrier
            // above ordered every consumer's partial writes before it) and, for
            // the last piece, acquires the other pieces for the merge below.
            int prev;
            asm volatile("atom.add.acq_rel.gpu.global.s32 %0, [%1], 1;"
                         : "=r"(prev)
                         : "l"(&p.counters[seg])
                         : "memory");
            last = prev == npieces - 1;
          }
          *merge_flag = last;
        }
        named_bar_sync(1, kConsumers);
        if (*merge_flag) {
          // Last piece in: merge all pieces of the segment.  Piece i was written
          // by CTA q = p_first + i into slot 2q (segment began at or before q's
          // range) or 2q+1 (it began inside q's range).
          auto piece_slot = [&](int i) {
            const int q = p_first + i;
            return seg_begin <= q * per_cta ? 2 * q : 2 * q + 1;
          };
          float4 acc[kElems4];
#pragma unroll
          for (int k4 = 0; k4 < kElems4; ++k4) acc[k4] = make_float4(0.f, 0.f, 0.f, 0.f);
          if constexpr (kTrans) {
            // One pass, no shared memory.  Thread t owns the kElems4 consecutive
            // outputs t * kElems4 ..: one row, so one lse and one running max /
            // rescaled sum per piece.  Each batch loads the lse and the partial O
            // of kPB pieces (16 float4 plus kPB lse, all independent), then folds
            // them in piece order, so a merge of n pieces costs about n / kPB L2
            // round trips in all.  Pieces without a visible key (lse = -inf;
            // their partial is 0/0) are skipped.
            static_assert(kD4 % kElems4 == 0, "a thread's merge outputs share one row");
            constexpr int kPB = 16 / kElems4;
            const int e0 = tid * kElems4;
            const int row = e0 / kD4;
            const int d40 = e0 - row * kD4;
            const bool mine = e0 < GH * kD4;
            float m_run = -INFINITY, s_run = 0.f;
            for (int q0 = 0; q0 < npieces; q0 += kPB) {
              float lse[kPB];
              float4 v[kPB][kElems4];
#pragma unroll
              for (int u = 0; u < kPB; ++u) {
                const bool in = mine && q0 + u < npieces;
                const long long base = in ? static_cast<long long>(piece_slot(q0 + u)) * GH + row : 0;
                lse[u] = in ? __ldcg(p.part_lse + base) : -INFINITY;
#pragma unroll
                for (int j = 0; j < kElems4; ++j)
                  v[u][j] = in ? __ldcg(reinterpret_cast<const float4*>(p.part_o) + base * kD4 +
                                        d40 + j)
                               : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int u = 0; u < kPB; ++u) {
                const float l = lse[u];
                if (l == -INFINITY) continue;
                float c = 1.f, w = 1.f;
                if (l > m_run) {
                  c = m_run == -INFINITY ? 0.f : fast_exp2(m_run - l);
                  m_run = l;
                } else {
                  w = fast_exp2(l - m_run);
                }
                s_run = s_run * c + w;
#pragma unroll
                for (int j = 0; j < kElems4; ++j) {
                  acc[j].x = acc[j].x * c + w * v[u][j].x;
                  acc[j].y = acc[j].y * c + w * v[u][j].y;
                  acc[j].z = acc[j].z * c + w * v[u][j].z;
                  acc[j].w = acc[j].w * c + w * v[u][j].w;
                }
              }
            }
            // No visible key in any piece: 0, the weighted sum of no pieces.
            const float inv = s_run > 0.f ? 1.f / s_run : 0.f;
            if (mine) {
#pragma unroll
              for (int j = 0; j < kElems4; ++j) {
                acc[j].x *= inv;
                acc[j].y *= inv;
                acc[j].z *= inv;
                acc[j].w *= inv;
                store4<E>(out_seg + row * p.out_stride_head + (d40 + j) * 4, acc[j]);
              }
            }
          } else {
            // Heads-as-M (G > 16): its main-loop state leaves no registers for
            // batches of O.  The lse of every (piece, row) of a chunk is loaded
            // at once (independent loads) into merge_w, then each row folds its
            // pieces in order into a running max and rescaled sum.  With few
            // pieces the lse values stay in merge_w for the weights below (no
            // second global read).
            const bool lse_cached = npieces <= kMergeChunk;
            for (int row = tid; row < GH; row += kConsumers) {
              row_base[row] = -INFINITY;
              row_l[row] = 0.f;
            }
            for (int c0 = 0; c0 < npieces; c0 += kMergeChunk) {
              const int nq = min(kMergeChunk, npieces - c0);
#pragma unroll 4
              for (int i = tid; i < nq * GH; i += kConsumers) {
                const int q = i / GH;
                merge_w[i] = __ldcg(p.part_lse + piece_slot(c0 + q) * GH + (i - q * GH));
              }
              named_bar_sync(1, kConsumers);
              for (int row = tid; row < GH; row += kConsumers) {
                float m = row_base[row], sum = row_l[row];
                for (int q = 0; q < nq; ++q) {
                  const float lse = merge_w[q * GH + row];
                  if (lse == -INFINITY) continue;
                  if (lse > m) {
                    sum = (m == -INFINITY ? 0.f : sum * fast_exp2(m - lse)) + 1.f;
                    m = lse;
                  } else {
                    sum += fast_exp2(lse - m);
                  }
                }
                row_base[row] = m;
                row_l[row] = sum;
              }
              named_bar_sync(1, kConsumers);
            }
            for (int row = tid; row < GH; row += kConsumers) {
              row_base[row] = row_base[row] == -INFINITY ? 0.f : row_base[row];
              row_l[row] = 1.f / row_l[row];
            }
            named_bar_sync(1, kConsumers);
            for (int c0 = 0; c0 < npieces; c0 += kMergeChunk) {
              const int nq = min(kMergeChunk, npieces - c0);
              for (int i = tid; i < kMergeChunk * GH; i += kConsumers) {
                const int q = i / GH;
                const int row = i - q * GH;
                float w = 0.f;
                if (q < nq) {
                  const float lse =
                      lse_cached ? merge_w[i] : __ldcg(p.part_lse + piece_slot(c0 + q) * GH + row);
                  if (lse != -INFINITY) w = fast_exp2(lse - row_base[row]) * row_l[row];
                }
                merge_w[i] = w;
              }
              named_bar_sync(1, kConsumers);
#pragma unroll
              for (int k4 = 0; k4 < kElems4; ++k4) {
                const int e = tid + k4 * kConsumers;
                if (e < GH * kD4) {
                  const int row = e / kD4;
                  const int d4 = e - row * kD4;
#pragma unroll 4
                  for (int q = 0; q < nq; ++q) {
                    const float w = merge_w[q * GH + row];
                    if (w == 0.f) continue;
                    const float4 v = __ldcg(reinterpret_cast<const float4*>(p.part_o) +
                                            (static_cast<long long>(piece_slot(c0 + q)) * GH +
                                             row) * kD4 + d4);
                    acc[k4].x += w * v.x;
                    acc[k4].y += w * v.y;
                    acc[k4].z += w * v.z;
                    acc[k4].w += w * v.w;
                  }
                }
              }
              named_bar_sync(1, kConsumers);
            }
#pragma unroll
            for (int k4 = 0; k4 < kElems4; ++k4) {
              const int e = tid + k4 * kConsumers;
              if (e < GH * kD4) {
                const int row = e / kD4;
                store4<E>(out_seg + row * p.out_stride_head + (e - row * kD4) * 4, acc[k4]);
              }
            }
          }
          if (tid == 0) p.counters[seg] = 0;
        }
      }
      named_bar_sync(1, kConsumers);
      seg_start = true;
    }
    cur.advance(len_s, B, HG, TT);
  }
}

// ------------------------------------------------------------------- host

struct WorkspaceLayout {
  size_t err_off, counters_off, lse_off, o_off, total;
};

// [0, 256): device error word.  Then the split partials, whose size depends only
// on (grid, query heads per segment = G * HB, head_dim) -- fixed for a model on
// a device -- and last the per-segment counters (num_seqs * kv_heads, at least
// the number of segments).  Counters go last so that a change
// of batch size never moves them onto bytes that held partials: counters past
// the previous batch were never written, the others were reset by the kernel.
static WorkspaceLayout workspace_layout(int num_seqs, int hkv, int group, int head_dim, int grid) {
  auto round256 = [](size_t x) { return (x + 255) / 256 * 256; };
  WorkspaceLayout w;
  size_t off = 0;
  w.err_off = off;
  off += 256;
  w.lse_off = off;
  off += round256(static_cast<size_t>(2) * grid * group * 4);
  w.o_off = off;
  off += round256(static_cast<size_t>(2) * grid * group * head_dim * 4);
  w.counters_off = off;
  off += round256(static_cast<size_t>(num_seqs) * hkv * 4);
  w.total = off;
  return w;
}

template <typename E, int D, int MT>
static int launch_decode_t(const CUtensorMap& kmap, const CUtensorMap& vmap,
                           const DecodeParams& p, int num_sms, int* grid_out, bool dry_run,
                           cudaStream_t stream) {
  const DecodeSmem L = decode_smem_layout<D, MT>(p.group, p.heads_per_tile, p.num_seqs);
  const int smem = L.total + 1024;
  const int fused = p.fuse_append ? 1 : 0;
  auto kern = fused ? paged_decode_kernel<E, D, MT, true> : paged_decode_kernel<E, D, MT, false>;
  static int configured_smem[2][64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && configured_smem[fused][dev] < smem) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return cuda_status(err, "cudaFuncSetAttribute(decode smem)");
    configured_smem[fused][dev] = smem;
  }
  int per_sm = 0;
  cudaError_t err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kDecThreads, smem);
  if (err != cudaSuccess) return cuda_status(err, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  if (per_sm < 1)
    return set_error(B200_ERR_UNSUPPORTED, "decode kernel does not fit on an SM (shared memory)");
  const int grid = num_sms * per_sm;
  // The workspace is sized for the largest grid of this instantiation (the
  // occupancy at batch size 1), so its layout does not move with the batch.
  const int smem_min = decode_smem_layout<D, MT>(p.group, p.heads_per_tile, 1).total + 1024;
  int per_sm_max = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm_max, kern, kDecThreads, smem_min);
  if (err != cudaSuccess) return cuda_status(err, "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  *grid_out = num_sms * (per_sm_max > per_sm ? per_sm_max : per_sm);
  if (dry_run) return B200_OK;
  // Programmatic stream serialization: the grid may be scheduled while the
  // previous kernel on the stream finishes (the kernel waits for it before any
  // global access), hiding the launch and set-up behind that kernel's tail.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t lerr = cudaLaunchKernelEx(&cfg, kern, kmap, vmap, p);
  if (lerr != cudaSuccess) return cuda_status(lerr, "paged_decode_kernel launch");
  return cuda_status(cudaGetLastError(), "paged_decode_kernel launch");
}

// Variant code per head group G: -1 (G <= 8) and -2 (G <= 16) use the
// transposed form; 2 (G <= 32) and 4 (G <= 64) put the heads on the M rows.
static int decode_variant(int group) {
  return group <= 8 ? -1 : (group <= 16 ? -2 : (group <= 32 ? 2 : 4));
}

// Kv heads per tile: 4 or 2 where the head-group geometry applies (transposed
// variants, G * HB <= 16 query heads per segment, head_dim 64/128, one page
// covering 64 / HB tokens), else 1.
static int decode_heads_per_tile(const b200_cache_desc* c, int group) {
  if (decode_variant(group) > 0) return 1;
  CacheTmaGeometry geo;
  for (int hb = 4; hb >= 2; hb /= 2)
    if (group * hb <= 16 && cache_head_group_geometry(c, hb, &geo)) return hb;
  return 1;
}

template <typename E, int D>
static int dispatch_mt(int mt, const CUtensorMap& kmap, const CUtensorMap& vmap,
                       const DecodeParams& p, int num_sms, int* grid, bool dry, cudaStream_t s) {
  switch (mt) {
    case -1: return launch_decode_t<E, D, -1>(kmap, vmap, p, num_sms, grid, dry, s);
    case -2: return launch_decode_t<E, D, -2>(kmap, vmap, p, num_sms, grid, dry, s);
    case 2: return launch_decode_t<E, D, 2>(kmap, vmap, p, num_sms, grid, dry, s);
    default: return launch_decode_t<E, D, 4>(kmap, vmap, p, num_sms, grid, dry, s);
  }
}

template <typename E>
static int dispatch_d(int d, int mt, const CUtensorMap& kmap, const CUtensorMap& vmap,
                      const DecodeParams& p, int num_sms, int* grid, bool dry, cudaStream_t s) {
  switch (d) {
    case 16: return dispatch_mt<E, 16>(mt, kmap, vmap, p, num_sms, grid, dry, s);
    case 32: return dispatch_mt<E, 32>(mt, kmap, vmap, p, num_sms, grid, dry, s);
    case 64: return dispatch_mt<E, 64>(mt, kmap, vmap, p, num_sms, grid, dry, s);
    default: return dispatch_mt<E, 128>(mt, kmap, vmap, p, num_sms, grid, dry, s);
  }
}

static int check_decode_args(const b200_cache_desc* c, const b200_decode_args* a) {
  if (c == nullptr || a == nullptr) return set_error(B200_ERR_INVALID, "null descriptor");
  if (c->num_layers <= 0 || c->num_blocks <= 0 || c->block_size <= 0 || c->num_kv_heads <= 0 ||
      c->head_dim <= 0)
    return set_error(B200_ERR_INVALID, "cache dimensions must be positive");
  if (c->dtype != B200_F16 && c->dtype != B200_BF16)
    return set_error(B200_ERR_UNSUPPORTED, "cache dtype must be float16 or bfloat16");
  if (c->head_dim != 16 && c->head_dim != 32 && c->head_dim != 64 && c->head_dim != 128)
    return set_error(B200_ERR_UNSUPPORTED, "head_dim must be one of 16, 32, 64, 128");
  if ((c->block_size & (c->block_size - 1)) != 0 || c->block_size > 256)
    return set_error(B200_ERR_UNSUPPORTED, "block_size must be a power of two <= 256");
  if (a->layer < 0 || a->layer >= c->num_layers)
    return set_error(B200_ERR_LAYER, "layer is out of range");
  if (a->num_seqs <= 0 || a->num_q_heads <= 0)
    return set_error(B200_ERR_INVALID, "query dimensions must be positive");
  if (a->num_seqs > kDecMaxSeqs)
    return set_error(B200_ERR_UNSUPPORTED, "decode batch is limited to 8192 sequences");
  if (a->num_q_heads % c->num_kv_heads != 0)
    return set_error(B200_ERR_INVALID, "num_heads must be divisible by num_kv_heads");
  if (a->num_q_heads / c->num_kv_heads > 64)
    return set_error(B200_ERR_UNSUPPORTED, "at most 64 query heads per kv head");
  if (a->table_width <= 0)
    return set_error(B200_ERR_INVALID, "block_tables must contain at least one logical block");
  const int64_t slots = static_cast<int64_t>(c->num_layers) * c->num_blocks * c->block_size;
  if (slots >= (1ll << 31)) return set_error(B200_ERR_UNSUPPORTED, "cache has more than 2^31 slots");
  if (static_cast<int64_t>(a->table_width) * c->block_size >= (1ll << 30))
    return set_error(B200_ERR_UNSUPPORTED, "block table capacity too large");
  if ((a->q_stride_seq | a->q_stride_head) & 1)
    return set_error(B200_ERR_INVALID, "query strides must be even");
  if ((a->out_stride_seq | a->out_stride_head) & 3)
    return set_error(B200_ERR_INVALID, "out strides must be multiples of 4 elements");
  return B200_OK;
}

size_t decode_workspace_bytes(const b200_cache_desc* c, const b200_decode_args* a) {
  clear_error();
  if (check_decode_args(c, a) != B200_OK) return 0;
  DeviceInfo info;
  if (current_device_info(&info) != B200_OK) return 0;
  const int group = a->num_q_heads / c->num_kv_heads;
  const int mt = decode_variant(group);
  const int hb = decode_heads_per_tile(c, group);
  CUtensorMap dummy;
  DecodeParams p{};
  p.group = group;
  p.heads_per_tile = hb;
  p.num_seqs = a->num_seqs;
  int grid = 0;
  int rc = c->dtype == B200_BF16
               ? dispatch_d<BF16>(c->head_dim, mt, dummy, dummy, p, info.num_sms, &grid, true, 0)
               : dispatch_d<Half>(c->head_dim, mt, dummy, dummy, p, info.num_sms, &grid, true, 0);
  if (rc != B200_OK) return 0;
  return workspace_layout(a->num_seqs, c->num_kv_heads, group * hb, c->head_dim, grid).total;
}

// Inputs of the fused new-token append (b200_paged_decode_append).
struct FusedAppend {
  const b200_decode_append_args* args;
  const void* key;
  const void* value;
  const void* cos;
  const void* sin;
  const void* slots;
};

static int launch_decode_common(const b200_cache_desc* c, const b200_decode_args* a,
                                const void* query, const void* block_tables,
                                const void* context_lens, void* out, void* workspace,
                                size_t workspace_bytes, const FusedAppend* f,
                                cudaStream_t stream) {
  int rc = check_decode_args(c, a);
  if (rc != B200_OK) return rc;
  if (f != nullptr) {
    const b200_decode_append_args* fa = f->args;
    if (fa == nullptr) return set_error(B200_ERR_INVALID, "null append descriptor");
    if (fa->rope != 0 && fa->rope != 1) return set_error(B200_ERR_INVALID, "rope must be 0 or 1");
    if (!f->key || !f->value || !f->slots)
      return set_error(B200_ERR_INVALID, "null key/value/slots pointer");
    // The new rows move as 16-byte vectors.
    if (((reinterpret_cast<uintptr_t>(f->key) | reinterpret_cast<uintptr_t>(f->value)) & 15) ||
        ((fa->k_stride_seq | fa->k_stride_head | fa->v_stride_seq | fa->v_stride_head) & 7))
      return set_error(B200_ERR_INVALID, "key/value rows must be 16-byte aligned");
    if (fa->rope) {
      if (!f->cos || !f->sin) return set_error(B200_ERR_INVALID, "rope needs cos and sin");
      // q fragments and cos/sin are read as aligned pairs of 16-bit elements.
      if (((reinterpret_cast<uintptr_t>(f->cos) | reinterpret_cast<uintptr_t>(f->sin)) & 15) ||
          ((fa->cos_stride_seq | fa->sin_stride_seq) & 7))
        return set_error(B200_ERR_INVALID, "cos/sin rows must be 16-byte aligned");
      // The rotated query is staged in `out` with 16-byte vectors.
      if (((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(out)) & 15) ||
          ((a->q_stride_seq | a->q_stride_head | a->out_stride_seq | a->out_stride_head) & 7))
        return set_error(B200_ERR_INVALID,
                         "with rope, query and out rows must be 16-byte aligned");
    }
  }
  if (!query || !block_tables || !context_lens || !out || !c->k_cache || !c->v_cache)
    return set_error(B200_ERR_INVALID, "null tensor pointer");
  if ((reinterpret_cast<uintptr_t>(query) & 3) || (reinterpret_cast<uintptr_t>(out) & 7))
    return set_error(B200_ERR_INVALID, "query must be 4-byte and out 8-byte aligned");
  DeviceInfo info;
  rc = current_device_info(&info);
  if (rc != B200_OK) return rc;
  const int group = a->num_q_heads / c->num_kv_heads;
  const int mt = decode_variant(group);
  const int hb = decode_heads_per_tile(c, group);
  CacheTmaGeometry geo;
  std::string why;
  if (hb > 1) {
    if (!cache_head_group_geometry(c, hb, &geo))
      return set_error(B200_ERR_UNSUPPORTED, "head-group geometry rejected");
  } else if (!cache_tma_geometry(c, kDecTile, &geo, &why)) {
    return set_error(B200_ERR_UNSUPPORTED, why);
  }
  CUtensorMap kmap, vmap;
  rc = encode_cache_tensor_map(c, c->k_cache, geo, &kmap);
  if (rc != B200_OK) return rc;
  rc = encode_cache_tensor_map(c, c->v_cache, geo, &vmap);
  if (rc != B200_OK) return rc;

  DecodeParams p{};
  p.q = query;
  p.out = out;
  p.tables = block_tables;
  p.lens = context_lens;
  p.q_stride_seq = a->q_stride_seq;
  p.q_stride_head = a->q_stride_head;
  p.out_stride_seq = a->out_stride_seq;
  p.out_stride_head = a->out_stride_head;
  p.table_stride = a->table_stride;
  p.layer_slot_base = static_cast<long long>(a->layer) * c->num_blocks * c->block_size;
  p.num_seqs = a->num_seqs;
  p.num_kv_heads = c->num_kv_heads;
  p.group = group;
  p.table_width = a->table_width;
  p.num_blocks = c->num_blocks;
  p.block_size = c->block_size;
  p.box_rows = geo.box_rows;
  p.sw_mask = geo.swizzle_bytes == 0 ? 0 : geo.swizzle_bytes / 16 - 1;
  p.heads_per_tile = hb;
  p.tile_tokens = kDecTile / hb;
  p.table64 = a->table_dtype == B200_I64;
  p.lens64 = a->lens_dtype == B200_I64;
  p.scale_log2 = a->scale * 1.4426950408889634f;
  if (f != nullptr) {
    p.fuse_append = 1;
    p.rope = f->args->rope;
    p.slots64 = f->args->slots_dtype == B200_I64;
    p.new_k = f->key;
    p.new_v = f->value;
    p.cos = f->cos;
    p.sin = f->sin;
    p.new_slots = f->slots;
    p.k_cache = c->k_cache;
    p.v_cache = c->v_cache;
    p.nk_stride_seq = f->args->k_stride_seq;
    p.nk_stride_head = f->args->k_stride_head;
    p.nv_stride_seq = f->args->v_stride_seq;
    p.nv_stride_head = f->args->v_stride_head;
    p.cos_stride = f->args->cos_stride_seq;
    p.sin_stride = f->args->sin_stride_seq;
    p.slots_per_layer = static_cast<long long>(c->num_blocks) * c->block_size;
  }

  int grid = 0;
  rc = c->dtype == B200_BF16
           ? dispatch_d<BF16>(c->head_dim, mt, kmap, vmap, p, info.num_sms, &grid, true, stream)
           : dispatch_d<Half>(c->head_dim, mt, kmap, vmap, p, info.num_sms, &grid, true, stream);
  if (rc != B200_OK) return rc;
  const WorkspaceLayout w =
      workspace_layout(a->num_seqs, c->num_kv_heads, group * hb, c->head_dim, grid);
  if (workspace == nullptr || workspace_bytes < w.total)
    return set_error(B200_ERR_WORKSPACE, "decode workspace missing or smaller than "
                                         "b200_paged_decode_workspace_bytes()");
  if (reinterpret_cast<uintptr_t>(workspace) & 255)
    return set_error(B200_ERR_WORKSPACE, "decode workspace must be 256-byte aligned");
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.err = reinterpret_cast<uint32_t*>(ws + w.err_off);
  p.counters = reinterpret_cast<int*>(ws + w.counters_off);
  p.part_lse = reinterpret_cast<float*>(ws + w.lse_off);
  p.part_o = reinterpret_cast<float*>(ws + w.o_off);
  return c->dtype == B200_BF16
             ? dispatch_d<BF16>(c->head_dim, mt, kmap, vmap, p, info.num_sms, &grid, false, stream)
             : dispatch_d<Half>(c->head_dim, mt, kmap, vmap, p, info.num_sms, &grid, false, stream);
}

int launch_paged_decode(const b200_cache_desc* c, const b200_decode_args* a, const void* query,
                        const void* block_tables, const void* context_lens, void* out,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return launch_decode_common(c, a, query, block_tables, context_lens, out, workspace,
                              workspace_bytes, nullptr, stream);
}

int launch_paged_decode_append(const b200_cache_desc* c, const b200_decode_args* a,
                               const b200_decode_append_args* fa, const void* query,
                               const void* key, const void* value, const void* cos,
                               const void* sin, const void* slots, const void* block_tables,
                               const void* context_lens, void* out, void* workspace,
                               size_t workspace_bytes, cudaStream_t stream) {
  const FusedAppend f{fa, key, value, cos, sin, slots};
  return launch_decode_common(c, a, query, block_tables, context_lens, out, workspace,
                              workspace_bytes, &f, stream);
}

// ------------------------------------------------------ allocation-free entry
//
// Some callers of this library cannot allocate device memory when they run
// attention: a plugin or custom operator inside a host framework's execute
// step (the host owns every buffer and forbids cudaMalloc there, which would
// also synchronise the device), or code running under a fixed memory budget.
// They pass only inputs and outputs; the split-KV scratch of the decode kernel
// then comes from this file-scope device array instead of a caller workspace.
//
// The array is kDecodeNoAllocScratchBytes (8 MiB) on every GPU that loads the
// library, kept until the process exits.  All calls share it and it keeps the
// last call's contents, so each call zeroes the parts that must start at zero
// (the error word and the split counters) before its launch, and calls whose
// executions overlap on the GPU (different streams, no ordering) race on it.
constexpr size_t kDecodeNoAllocScratchBytes = static_cast<size_t>(8) << 20;
static __device__ __align__(256) uint8_t g_decode_noalloc_scratch[kDecodeNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
// Device address of the array per device index, with the context it was
// resolved in: a different current context on that device (after
// cudaDeviceReset, or a context the caller made with the driver API) resolves
// it again instead of reusing a stale address.
struct NoAllocAddress {
  CUcontext ctx = nullptr;
  void* ptr = nullptr;
};
NoAllocAddress g_noalloc_addr[64];
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn g_ctx_get_current = nullptr;
}  // namespace

// Host code may not use the array's name as a device address; resolve it once
// per device (and context), with that device current.
static int noalloc_scratch_address(void** out) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) return cuda_status(err, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return set_error(B200_ERR_UNSUPPORTED, "device index >= 64");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_ctx_get_current == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    err = cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q);
    if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return set_error(B200_ERR_CUDA, "cuCtxGetCurrent entry point unavailable");
    g_ctx_get_current = reinterpret_cast<CtxGetCurrentFn>(fn);
  }
  // cudaGetDevice does not create the primary context; a runtime call that
  // needs one does, so resolve the symbol first when nothing is current yet.
  CUcontext ctx = nullptr;
  if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
  NoAllocAddress& slot = g_noalloc_addr[dev];
  if (slot.ptr == nullptr || ctx == nullptr || slot.ctx != ctx) {
    void* ptr = nullptr;
    err = cudaGetSymbolAddress(&ptr, g_decode_noalloc_scratch);
    if (err != cudaSuccess) return cuda_status(err, "cudaGetSymbolAddress(decode scratch)");
    if (g_ctx_get_current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    slot.ctx = ctx;
    slot.ptr = ptr;
  }
  *out = slot.ptr;
  return B200_OK;
}

size_t decode_noalloc_scratch_bytes() { return kDecodeNoAllocScratchBytes; }

// The error word sits at offset 0 of every workspace layout, so it is the
// array's first 4 bytes whatever the shape of the last call.
int decode_noalloc_error_word(uint32_t** out) {
  if (out == nullptr) return set_error(B200_ERR_INVALID, "error_word_out must not be NULL");
  void* scratch = nullptr;
  const int rc = noalloc_scratch_address(&scratch);
  if (rc != B200_OK) return rc;
  *out = static_cast<uint32_t*>(scratch);
  return B200_OK;
}

int launch_paged_decode_noalloc(const b200_cache_desc* c, const b200_decode_args* a,
                                const void* query, const void* block_tables,
                                const void* context_lens, void* out, cudaStream_t stream) {
  int rc = check_decode_args(c, a);
  if (rc != B200_OK) return rc;
  DeviceInfo info;
  rc = current_device_info(&info);
  if (rc != B200_OK) return rc;
  const int group = a->num_q_heads / c->num_kv_heads;
  const int mt = decode_variant(group);
  const int hb = decode_heads_per_tile(c, group);
  CUtensorMap unused;
  DecodeParams probe{};
  probe.group = group;
  probe.heads_per_tile = hb;
  probe.num_seqs = a->num_seqs;
  int grid = 0;
  rc = c->dtype == B200_BF16
           ? dispatch_d<BF16>(c->head_dim, mt, unused, unused, probe, info.num_sms, &grid, true, stream)
           : dispatch_d<Half>(c->head_dim, mt, unused, unused, probe, info.num_sms, &grid, true, stream);
  if (rc != B200_OK) return rc;
  const WorkspaceLayout w =
      workspace_layout(a->num_seqs, c->num_kv_heads, group * hb, c->head_dim, grid);
  if (w.total > kDecodeNoAllocScratchBytes)
    return set_error(B200_ERR_WORKSPACE,
                     "this decode shape needs " + std::to_string(w.total) +
                         " bytes of split scratch, more than the 8 MiB static scratch of "
                         "b200_paged_decode_noalloc; use b200_paged_decode with a workspace");
  void* scratch = nullptr;
  rc = noalloc_scratch_address(&scratch);
  if (rc != B200_OK) return rc;
  uint8_t* base = static_cast<uint8_t*>(scratch);
  cudaError_t err = cudaMemsetAsync(base + w.err_off, 0, 256, stream);
  if (err != cudaSuccess) return cuda_status(err, "cudaMemsetAsync(scratch error word)");
  err = cudaMemsetAsync(base + w.counters_off, 0, w.total - w.counters_off, stream);
  if (err != cudaSuccess) return cuda_status(err, "cudaMemsetAsync(scratch counters)");
  return launch_paged_decode(c, a, query, block_tables, context_lens, out, scratch,
                             kDecodeNoAllocScratchBytes, stream);
}

}  // namespace b200
