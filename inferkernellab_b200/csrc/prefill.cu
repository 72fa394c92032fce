// Ragged causal prefill attention over the paged KV cache, sm_100a.
//
// One CTA = (sequence b, query head h, tile of 64 query tokens).  Warp 4 is the
// TMA producer: it streams 64-token K/V tiles of kv head h / G, pages looked
// up in block_tables[b], through a STAGES-deep shared-memory ring.  Warps 0..3
// each own 16 query rows and run S = Q K^T, the causal mask, a base-2 online
// softmax and O += P V on mma.sync m16n8k16 with fp32 accumulation.  Key tiles
// past the tile's last query position are never loaded; 16-key groups past a
// warp's last row are skipped.
//
// Semantics follow the reference's paged_prefill_attention_sdpa
// (src/inferkernellab/attention.py:230-321): query token t of sequence b sits at
// logical position starts[b] + t and attends keys 0 .. starts[b] + t; keys at or
// past context_lens[b] are masked and their V rows zeroed (the reference's
// masked_fill at :301-305); in the padded layout, rows t >= ends-starts attend
// key 0 only (:313).
#include <math.h>

#include "../../include/b200_paged_attn.h"
#include "attn_core.cuh"
#include "common.cuh"
#include "host_common.h"
#include "prefill.h"
#include "prefill_params.h"

namespace b200 {

constexpr int kPreConsumerWarps = 4;
constexpr int kPreThreads = (kPreConsumerWarps + 1) * 32;
constexpr int kPreRows = kPreConsumerWarps * 16;  // query tokens per CTA

template <int D>
struct PrefillShape : KvTileShape<D> {
  static constexpr int kStages = D >= 128 ? 3 : 4;
};

template <int D>
__host__ __device__ inline int prefill_smem_bytes(int num_seqs, int packed) {
  using S = PrefillShape<D>;
  int off = S::kStages * 2 * S::kTileBytes;
  off += 3 * S::kStages * 8;                       // full, empty, masks
  off += 16;                                       // flags
  off += kTableWindow * 4;                         // producer's block-table window
  if (packed) off += (num_seqs + 1) * 4 + (kPreThreads / 32) * 4;  // tile prefix + scan
  return off;
}

template <typename E, int D>
__global__ void __launch_bounds__(kPreThreads, 2)
    paged_prefill_kernel(const __grid_constant__ CUtensorMap kmap,
                         const __grid_constant__ CUtensorMap vmap, const PrefillParams p) {
  using S = PrefillShape<D>;
  using T = typename E::T;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  int off = kStages * 2 * S::kTileBytes;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + off);
  uint64_t* empty_bar = full_bar + kStages;
  uint64_t* stage_mask = empty_bar + kStages;
  off += 3 * kStages * 8;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + off);
  off += 16;
  int* table_s = reinterpret_cast<int*>(smem + off);
  off += kTableWindow * 4;
  int* begin_s = reinterpret_cast<int*>(smem + off);
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
      mbar_init(&empty_bar[s], kPreConsumerWarps);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }

  // ---- which (sequence, query tile) this CTA owns ----
  int b = 0, qt = 0;
  if (!p.packed) {
    const int tiles = (p.max_query_len + kPreRows - 1) / kPreRows;
    b = blockIdx.x / tiles;
    qt = tiles - 1 - (blockIdx.x - b * tiles);  // heaviest tile of each sequence first
  } else {
    const int chunk = (B + kPreThreads - 1) / kPreThreads;
    const int lo = min(B, tid * chunk);
    const int hi = min(B, lo + chunk);
    int sum = 0;
    for (int i = lo; i < hi; ++i) {
      const long long n = p.cu_seqlens[i + 1] - p.cu_seqlens[i];
      sum += n > 0 ? static_cast<int>((n + kPreRows - 1) / kPreRows) : 0;
    }
    int total_tiles = 0;
    int acc = block_exclusive_scan<kPreThreads>(sum, scan_s, &total_tiles);
    for (int i = lo; i < hi; ++i) {
      begin_s[i] = acc;
      const long long n = p.cu_seqlens[i + 1] - p.cu_seqlens[i];
      acc += n > 0 ? static_cast<int>((n + kPreRows - 1) / kPreRows) : 0;
    }
    if (tid == 0) begin_s[B] = total_tiles;
    __syncthreads();
    const int x = blockIdx.x;
    if (x >= begin_s[B]) return;
    int lo2 = 0, hi2 = B;
    while (hi2 - lo2 > 1) {
      const int mid = (lo2 + hi2) >> 1;
      if (begin_s[mid] <= x) lo2 = mid; else hi2 = mid;
    }
    b = lo2;
    const int tiles = begin_s[b + 1] - begin_s[b];
    qt = tiles - 1 - (x - begin_s[b]);
  }
  __syncthreads();

  const long long start_b = load_index(p.starts, b, p.index64);
  long long end_b = load_index(p.ends, b, p.index64);
  long long len_b = end_b - start_b;
  if (start_b < 0 || len_b <= 0) len_b = 0;
  const long long key_end = end_b < cap ? end_b : cap;  // real keys are < key_end
  const int t0 = qt * kPreRows;
  // Rows of this tile that exist: padded layout has max_query_len rows per
  // sequence, packed layout has len_b.
  const long long rows_here = p.packed ? len_b : p.max_query_len;
  // Keys needed: up to the last valid query's position, at least key 0 when a
  // padding row exists in the tile.
  long long kmax = 0;
  if (t0 < len_b) kmax = start_b + min(static_cast<long long>(t0 + kPreRows), len_b);
  if (!p.packed && t0 + kPreRows > len_b && t0 < rows_here && kmax < 1) kmax = 1;
  if (kmax > key_end) kmax = key_end;
  const int n_ktiles = static_cast<int>((kmax + kKvTile - 1) / kKvTile);

  if (warp == kPreConsumerWarps) {
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
      uint8_t* kdst = smem + s * 2 * S::kTileBytes;
      issue_kv_tile<D>(&kmap, &vmap, p.src, win, b, row_pages, hkv, tok0, ntok, kdst,
                       kdst + S::kTileBytes, &full_bar[s], &stage_mask[s], p.err, lane);
      ++issued;
    }
    if (lane == 0) drain_stages<kStages>(full_bar, issued, p.err);
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int g = lane >> 2;
  const int tq = lane & 3;
  const int ta = t0 + warp * 16 + g;  // query token of fragment row g
  const int tb = ta + 8;              // ... of row g + 8
  auto row_limit = [&](long long t) -> int {
    if (t < len_b) return static_cast<int>(min(start_b + t + 1, key_end));
    if (!p.packed && t < rows_here) return 1;  // padding row: key 0 only
    return 0;                                  // row does not exist
  };
  const int lim0 = row_limit(ta);
  const int lim1 = row_limit(tb);
  auto q_row = [&](long long t, int lim) -> const T* {
    if (lim == 0) return nullptr;
    const T* base = reinterpret_cast<const T*>(p.q);
    if (p.packed)
      return base + (p.cu_seqlens[b] + t) * p.q_stride_token + h * p.q_stride_head;
    return base + b * p.q_stride_seq + h * p.q_stride_head + t * p.q_stride_token;
  };
  uint32_t qf[D / 16][4];
  load_q_frag<E, D>(qf, q_row(ta, lim0), q_row(tb, lim1), tq);
  float o[D / 8][4];
#pragma unroll
  for (int i = 0; i < D / 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_r[2] = {-INFINITY, -INFINITY};
  float l_r[2] = {0.f, 0.f};
  // Warp-uniform last key any of this warp's rows may see.
  int wlim = max(lim0, lim1);
  wlim = max(wlim, __shfl_xor_sync(0xffffffffu, wlim, 1));
  wlim = max(wlim, __shfl_xor_sync(0xffffffffu, wlim, 2));
  wlim = max(wlim, __shfl_xor_sync(0xffffffffu, wlim, 4));
  wlim = max(wlim, __shfl_xor_sync(0xffffffffu, wlim, 8));
  wlim = max(wlim, __shfl_xor_sync(0xffffffffu, wlim, 16));
  const uint32_t sw = static_cast<uint32_t>(p.sw_mask);
  const uint32_t smem_base = smem_u32(smem);
  bool aborted = false;
  for (int it = 0; it < n_ktiles; ++it) {
    const int s = it % kStages;
    const uint32_t k = static_cast<uint32_t>(it / kStages);
    if (!mbar_wait_bounded(&full_bar[s], k & 1u, abort_flag, p.err, kErrWaitFull)) {
      aborted = true;
      break;
    }
    const uint64_t tmask = stage_mask[s];
    const uint32_t kbase = smem_base + s * 2 * S::kTileBytes;
    const uint32_t vbase = kbase + S::kTileBytes;
#pragma unroll
    for (int gi = 0; gi < kKvTile / 16; ++gi) {
      const int key0 = it * kKvTile + gi * 16;
      const uint32_t gmask = static_cast<uint32_t>(tmask >> (gi * 16)) & 0xffffu;
      if (gmask == 0 || key0 >= wlim) continue;
      attend16<E, D, true>(qf, o, m_r, l_r, kbase, vbase, gi * 16, gmask, key0, lim0, lim1,
                           p.scale_log2, sw, lane);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty_bar[s]);
  }
  if (aborted) return;
  const float l0 = quad_sum(l_r[0]);
  const float l1 = quad_sum(l_r[1]);
  auto out_row = [&](long long t) -> T* {
    T* base = reinterpret_cast<T*>(p.out);
    if (p.packed) return base + (p.cu_seqlens[b] + t) * p.o_stride_token + h * p.o_stride_head;
    return base + b * p.o_stride_seq + h * p.o_stride_head + t * p.o_stride_token;
  };
  if (lim0 > 0) {
    T* dst = out_row(ta) + 2 * tq;
    const float inv = 1.f / l0;
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
      *reinterpret_cast<uint32_t*>(dst + i * 8) = pack2<E>(o[i][0] * inv, o[i][1] * inv);
  }
  if (lim1 > 0) {
    T* dst = out_row(tb) + 2 * tq;
    const float inv = 1.f / l1;
#pragma unroll
    for (int i = 0; i < D / 8; ++i)
      *reinterpret_cast<uint32_t*>(dst + i * 8) = pack2<E>(o[i][2] * inv, o[i][3] * inv);
  }
}

template <typename E, int D>
static int launch_prefill_t(const CUtensorMap& kmap, const CUtensorMap& vmap,
                            const PrefillParams& p, dim3 grid, cudaStream_t stream) {
  const int smem = prefill_smem_bytes<D>(p.num_seqs, p.packed) + 1024;
  auto kern = paged_prefill_kernel<E, D>;
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && configured[dev] < smem) {
    cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (err != cudaSuccess) return cuda_status(err, "cudaFuncSetAttribute(prefill smem)");
    configured[dev] = smem;
  }
  kern<<<grid, kPreThreads, smem, stream>>>(kmap, vmap, p);
  return cuda_status(cudaGetLastError(), "paged_prefill_kernel launch");
}

template <typename E>
static int prefill_dispatch_d(int d, const CUtensorMap& kmap, const CUtensorMap& vmap,
                              const PrefillParams& p, dim3 grid, cudaStream_t s) {
  switch (d) {
    case 16: return launch_prefill_t<E, 16>(kmap, vmap, p, grid, s);
    case 32: return launch_prefill_t<E, 32>(kmap, vmap, p, grid, s);
    case 64: return launch_prefill_t<E, 64>(kmap, vmap, p, grid, s);
    default: return launch_prefill_t<E, 128>(kmap, vmap, p, grid, s);
  }
}

int launch_paged_prefill(const b200_cache_desc* c, const b200_prefill_args* a, const void* query,
                         const void* block_tables, const void* query_starts,
                         const void* context_lens, const int32_t* cu_seqlens_q, void* out,
                         uint32_t* error_word, cudaStream_t stream) {
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
  if (a->num_seqs <= 0 || a->num_q_heads <= 0 || a->num_q_heads % c->num_kv_heads != 0)
    return set_error(B200_ERR_INVALID, "num_heads must be positive and divisible by num_kv_heads");
  if (a->num_seqs > kPreMaxSeqs)
    return set_error(B200_ERR_UNSUPPORTED, "prefill batch is limited to 8192 sequences");
  if (a->table_width <= 0)
    return set_error(B200_ERR_INVALID, "block_tables must contain at least one logical block");
  if (a->query_layout != 0 && a->query_layout != 1)
    return set_error(B200_ERR_INVALID, "query_layout must be 0 (padded) or 1 (packed)");
  if (a->query_layout == 1 && cu_seqlens_q == nullptr)
    return set_error(B200_ERR_INVALID, "packed prefill needs cu_seqlens_q");
  if (a->max_query_len <= 0 && a->query_layout == 0)
    return set_error(B200_ERR_INVALID, "query width must be positive");
  if (!query || !out || !block_tables || !query_starts || !context_lens)
    return set_error(B200_ERR_INVALID, "null tensor pointer");
  if ((a->q_stride_seq | a->q_stride_head | a->q_stride_token | a->o_stride_seq |
       a->o_stride_head | a->o_stride_token) & 1)
    return set_error(B200_ERR_INVALID, "query/out strides must be even");
  if ((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(out)) & 3)
    return set_error(B200_ERR_INVALID, "query/out must be 4-byte aligned");
  const int64_t slots = static_cast<int64_t>(c->num_layers) * c->num_blocks * c->block_size;
  if (slots >= (1ll << 31)) return set_error(B200_ERR_UNSUPPORTED, "cache has more than 2^31 slots");

  CacheTmaGeometry geo;
  std::string why;
  if (!cache_tma_geometry(c, kKvTile, &geo, &why)) return set_error(B200_ERR_UNSUPPORTED, why);
  CUtensorMap kmap, vmap;
  int rc = encode_cache_tensor_map(c, c->k_cache, geo, &kmap);
  if (rc != B200_OK) return rc;
  rc = encode_cache_tensor_map(c, c->v_cache, geo, &vmap);
  if (rc != B200_OK) return rc;

  PrefillParams p{};
  p.q = query;
  p.out = out;
  p.starts = query_starts;
  p.ends = context_lens;
  p.cu_seqlens = cu_seqlens_q;
  p.err = error_word;
  p.src.tables = block_tables;
  p.src.table_stride = a->table_stride;
  p.src.layer_slot_base = static_cast<long long>(a->layer) * c->num_blocks * c->block_size;
  p.src.table64 = a->table_dtype == B200_I64;
  p.src.num_blocks = c->num_blocks;
  p.src.block_size = c->block_size;
  p.src.box_rows = geo.box_rows;
  p.q_stride_seq = a->q_stride_seq;
  p.q_stride_head = a->q_stride_head;
  p.q_stride_token = a->q_stride_token;
  p.o_stride_seq = a->o_stride_seq;
  p.o_stride_head = a->o_stride_head;
  p.o_stride_token = a->o_stride_token;
  p.num_seqs = a->num_seqs;
  p.group = a->num_q_heads / c->num_kv_heads;
  p.num_kv_heads = c->num_kv_heads;
  p.packed = a->query_layout;
  p.max_query_len = a->max_query_len;
  p.index64 = a->index_dtype == B200_I64;
  p.table_width = a->table_width;
  p.sw_mask = geo.swizzle_bytes == 0 ? 0 : geo.swizzle_bytes / 16 - 1;
  p.scale_log2 = a->scale * 1.4426950408889634f;

  if (a->kernel != B200_PREFILL_AUTO && a->kernel != B200_PREFILL_TCGEN05 &&
      a->kernel != B200_PREFILL_MMA_SYNC)
    return set_error(B200_ERR_INVALID, "unknown prefill kernel selector");
  // tcgen05 kernel: head_dim 64/128, 128-byte swizzled cache tiles, 16-byte
  // aligned query/output rows (it moves rows with 16-byte vectors).
  const long long row_bits = a->q_stride_head | a->q_stride_token | a->o_stride_head |
                             a->o_stride_token |
                             (a->query_layout == 0 ? (a->q_stride_seq | a->o_stride_seq) : 0);
  const bool pow2_group = (p.group & (p.group - 1)) == 0;
  const bool tc_ok = (c->head_dim == 64 || c->head_dim == 128) && p.group <= 64 && pow2_group &&
                     a->scale > 0.f &&
                     geo.swizzle_bytes == 128 &&
                     geo.chunk_bytes == 128 && (row_bits & 7) == 0 &&
                     ((reinterpret_cast<uintptr_t>(query) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  if (a->kernel == B200_PREFILL_TCGEN05 && !tc_ok)
    return set_error(B200_ERR_UNSUPPORTED,
                     "tcgen05 prefill needs head_dim 64/128, block_size >= 8, a power-of-two number "
                     "(<= 64) of query heads per kv head, a positive scale and 16-byte aligned "
                     "query/output rows");
  if (tc_ok && a->kernel != B200_PREFILL_MMA_SYNC) {
    const int qb = prefill_tc_query_block(p.group);
    long long items;
    if (a->query_layout == 0) {
      items = static_cast<long long>(a->num_seqs) * ((a->max_query_len + qb - 1) / qb);
    } else {
      if (a->total_query_tokens <= 0) return B200_OK;
      items = (a->total_query_tokens + qb - 1) / qb + a->num_seqs;
    }
    const long long tx = items * c->num_kv_heads;
    if (tx > 0x7fffffffLL) return set_error(B200_ERR_UNSUPPORTED, "prefill grid too large");
    // The query's TMA map: box {64 elements, heads per tile, tokens per tile}.
    const uint32_t ht = static_cast<uint32_t>(prefill_tc_query_heads_per_tile(p.group));
    const uint32_t tpt = static_cast<uint32_t>(kTcRows) / ht;
    // The query's and the output's TMA maps: box {64 elements, heads per tile,
    // tokens per tile (, 1 sequence)}.
    CUtensorMap qmap, omap;
    for (int which = 0; which < 2 && rc == B200_OK; ++which) {
      const void* base = which == 0 ? query : out;
      const int64_t sh = which == 0 ? a->q_stride_head : a->o_stride_head;
      const int64_t st = which == 0 ? a->q_stride_token : a->o_stride_token;
      const int64_t ss = which == 0 ? a->q_stride_seq : a->o_stride_seq;
      CUtensorMap* dst = which == 0 ? &qmap : &omap;
      if (a->query_layout == 1) {
        const uint64_t dims[3] = {static_cast<uint64_t>(c->head_dim),
                                  static_cast<uint64_t>(a->num_q_heads),
                                  static_cast<uint64_t>(a->total_query_tokens)};
        const uint64_t strides[2] = {static_cast<uint64_t>(sh) * 2, static_cast<uint64_t>(st) * 2};
        const uint32_t box[3] = {64u, ht, tpt};
        rc = encode_tensor_map_16b(base, 3, dims, strides, box, c->dtype, dst);
      } else {
        const uint64_t dims[4] = {static_cast<uint64_t>(c->head_dim),
                                  static_cast<uint64_t>(a->num_q_heads),
                                  static_cast<uint64_t>(a->max_query_len),
                                  static_cast<uint64_t>(a->num_seqs)};
        const uint64_t strides[3] = {static_cast<uint64_t>(sh) * 2, static_cast<uint64_t>(st) * 2,
                                     static_cast<uint64_t>(ss) * 2};
        const uint32_t box[4] = {64u, ht, tpt, 1u};
        rc = encode_tensor_map_16b(base, 4, dims, strides, box, c->dtype, dst);
      }
    }
    if (rc != B200_OK) return rc;
    return launch_prefill_tc(kmap, vmap, qmap, omap, p, c->head_dim, c->dtype == B200_BF16,
                             static_cast<unsigned>(tx), 1u, stream);
  }

  long long gx;
  if (a->query_layout == 0) {
    gx = static_cast<long long>(a->num_seqs) * ((a->max_query_len + kPreRows - 1) / kPreRows);
  } else {
    if (a->total_query_tokens <= 0) return B200_OK;
    gx = (a->total_query_tokens + kPreRows - 1) / kPreRows + a->num_seqs;
  }
  if (gx > 0x7fffffffLL) return set_error(B200_ERR_UNSUPPORTED, "prefill grid too large");
  dim3 grid(static_cast<unsigned>(gx), static_cast<unsigned>(a->num_q_heads));
  return c->dtype == B200_BF16 ? prefill_dispatch_d<BF16>(c->head_dim, kmap, vmap, p, grid, stream)
                               : prefill_dispatch_d<Half>(c->head_dim, kmap, vmap, p, grid, stream);
}

}  // namespace b200
