// Row movers: the selected-row gather from pinned host memory into HBM (mskv_uva_gather,
// mskv_gather) and the contiguous row copies behind the paged append and the host write-back
// (mskv_copy_rows).
//
// Design (B200): the work is tiles of rows of one (b, h) segment; a CTA takes tiles in a
// grid-stride loop (a bounded grid for moves that touch host memory, see launch_move).  For
// each tile the first threads resolve the source/destination byte offsets (index list, ring,
// page table, bounds) into shared memory once per row; then all 256 threads stream the tile
// as VEC-byte chunks with UNROLL independent loads in flight per thread for K and for V
// before any store.  The offsets of the CTA's next tile are resolved while the current
// tile's loads are in flight (two offset sets), so the index reads do not sit between tiles.
// Consecutive threads take consecutive 16-byte chunks of a row, so one half-warp reads one
// 256-byte bf16 row (two aligned 128-byte PCIe read requests) and the stores to HBM are
// fully coalesced.  Rows that are invalid (index out of range, unmapped page) are skipped
// (gathered rows zero-filled) and reported through the status word; nothing ever reads or
// writes outside the described buffers.
#include "common.cuh"

namespace mskv {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;
constexpr int kMaxRowsPerCta = 256;

struct MoveDev {
  RowsDev src, dst;
  const void* idx;          // gather: index list (int32/int64); copy: NULL
  int64_t idx_sb, idx_sh;
  const int32_t* counts;
  int64_t cnt_sb, cnt_sh;
  int64_t row_bytes;
  uint32_t* status;
  int32_t idx64;
  int32_t batch, heads;
  int32_t rows_max;         // rows per segment (upper bound)
  int32_t rows_per_cta;
  int32_t tiles;            // ceil(rows_max / rows_per_cta)
  int32_t chunk_shift;      // log2(row_bytes / VEC) or -1
  int32_t zero_invalid;     // zero-fill destination rows whose source is invalid
  int32_t work;             // tiles in all segments (segments x tiles)
};

// Resolves the source/destination byte offsets of tile w's rows into s_src / s_dst (one row per
// thread); returns the tile's row count (0: the tile holds no rows), the same in every thread.
__device__ __forceinline__ int resolve_tile(const MoveDev& a, int w, int64_t* s_src, int64_t* s_dst) {
  const int seg = w / a.tiles;
  const int tile = w - seg * a.tiles;
  const int b = seg / a.heads;
  const int h = seg - b * a.heads;
  int count = a.rows_max;
  if (a.counts) {
    count = a.counts[(int64_t)b * a.cnt_sb + (int64_t)h * a.cnt_sh];
    if (count > a.rows_max) count = a.rows_max;
  }
  const int r0 = tile * a.rows_per_cta;
  if (r0 >= count) return 0;
  const int nrows = min(a.rows_per_cta, count - r0);
  if (threadIdx.x < nrows) {
    const int i = r0 + threadIdx.x;
    uint32_t why = 0;
    int64_t st;
    if (a.idx) {
      const int64_t o = (int64_t)b * a.idx_sb + (int64_t)h * a.idx_sh + i;
      st = a.idx64 ? static_cast<const int64_t*>(a.idx)[o] : (int64_t) static_cast<const int32_t*>(a.idx)[o];
    } else {
      st = (a.src.tok0 ? a.src.tok0[b] : 0) + (int64_t)i;
    }
    const int64_t dt = (a.dst.tok0 ? a.dst.tok0[b] : 0) + (int64_t)i;
    int64_t so = rows_offset(a.src, b, h, st, &why, MSKV_STATUS_INDEX_OOB);
    const int64_t dof = rows_offset(a.dst, b, h, dt, &why, MSKV_STATUS_DST_OOB);
    if (so < 0 && !a.zero_invalid) so = -1;
    s_src[threadIdx.x] = so;
    s_dst[threadIdx.x] = dof;
    if (why && a.status) atomicOr(a.status, why);
  }
  return nrows;
}

template <int VEC>
__global__ void __launch_bounds__(kThreads) move_rows_kernel(const MoveDev a) {
  using V = typename Vec<VEC>::T;
  // Two sets of row offsets: the next tile's are resolved (its index loads issued and waited
  // for) while the current tile's row loads are in flight.
  __shared__ int64_t s_src[2][kMaxRowsPerCta];
  __shared__ int64_t s_dst[2][kMaxRowsPerCta];

  const int64_t chunks = a.row_bytes / VEC;
  const char* __restrict__ sk = a.src.base_k;
  const char* __restrict__ sv = a.src.base_v;
  char* __restrict__ dk = const_cast<char*>(a.dst.base_k);
  char* __restrict__ dv = const_cast<char*>(a.dst.base_v);
  const bool has_v = sv != nullptr;

  // Grid-stride loop over the tiles: the grid may be smaller than the work (see launch_move).
  int w = blockIdx.x;
  int nrows = 0;
  while (w < a.work && (nrows = resolve_tile(a, w, s_src[0], s_dst[0])) == 0) w += gridDim.x;
  int buf = 0;
  __syncthreads();
  while (w < a.work) {
    const int64_t total = (int64_t)nrows * chunks;
    int wn = w + (int)gridDim.x, nn = 0;
    bool next_resolved = false;
    for (int64_t base = threadIdx.x; base < total; base += (int64_t)kThreads * kUnroll) {
      V rk[kUnroll], rv[kUnroll];
      int64_t dofs[kUnroll];
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        const int64_t item = base + (int64_t)u * kThreads;
        dofs[u] = -1;
        rk[u] = V{};
        rv[u] = V{};
        if (item < total) {
          const int64_t r = a.chunk_shift >= 0 ? (item >> a.chunk_shift) : (item / chunks);
          const int64_t c = item - r * chunks;
          const int64_t so = s_src[buf][r];
          const int64_t dof = s_dst[buf][r];
          if (dof >= 0 && (so >= 0 || a.zero_invalid)) {
            dofs[u] = dof + c * VEC;
            if (so >= 0) {
              rk[u] = *reinterpret_cast<const V*>(sk + so + c * VEC);
              if (has_v) rv[u] = *reinterpret_cast<const V*>(sv + so + c * VEC);
            }
          }
        }
      }
      if (!next_resolved) {            // while this round's loads are in flight (uniform)
        while (wn < a.work && (nn = resolve_tile(a, wn, s_src[buf ^ 1], s_dst[buf ^ 1])) == 0)
          wn += gridDim.x;
        next_resolved = true;
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (dofs[u] >= 0) {
          *reinterpret_cast<V*>(dk + dofs[u]) = rk[u];
          if (has_v) *reinterpret_cast<V*>(dv + dofs[u]) = rv[u];
        }
      }
    }
    if (!next_resolved)
      while (wn < a.work && (nn = resolve_tile(a, wn, s_src[buf ^ 1], s_dst[buf ^ 1])) == 0)
        wn += gridDim.x;
    // the next tile's offsets are visible, and every reader of this tile's set is done with it
    __syncthreads();
    w = wn;
    nrows = nn;
    buf ^= 1;
  }
}

// ---------------------------------------------------------------------------------------
// Bulk-copy row mover, for moves that read or write host memory (the UVA gather and the
// write-back), when every row starts on a 16-byte boundary and is a multiple of 16 bytes.
//
// Used for rows of 1 KiB and more (kBulkMinRow).
// Each warp runs its own pipeline over tiles of up to 32 rows of one segment: the lanes resolve
// their rows' offsets (one row per lane), lane 0 issues one 1-D bulk copy per row
// (cp.async.bulk, no multicast) into one of the warp's two shared-memory banks, completing on
// that bank's mbarrier, and, once the bank is full, one bulk copy per row from shared memory to
// the destination.  While one bank drains, the next tile's rows are already in flight into the
// other.  A row is then a single copy instruction, so a transfer ramps up faster than with
// 16-byte loads, most visibly for small transfers.  Every mbarrier wait is bounded: after the
// limit the warp sets MSKV_STATUS_TIMEOUT, waits (bounded too) for its other bank and its
// stores, and stops.
constexpr int kBulkWarps = 4;
constexpr int kBulkBank = 16 * 1024;                 // bytes per bank per warp
constexpr int kBulkMaxRow = kBulkBank / 2;           // K and V rows of one tile share a bank
// Rows below this size move faster as 16-byte loads: the decode step's 256-byte (one head) rows
// measured 0.907 of the link with bulk copies against 0.919 with loads, while whole-token rows
// (1-2 KiB) gain from them, most in small transfers and in write-back.
constexpr int kBulkMinRow = 1024;

// One tile's rows as the warp sees them: lane i holds row i's offsets (valid for i < n).
struct BulkTile {
  int64_t so, dof;
  int n;
};

template <bool HAS_V>
__global__ void __launch_bounds__(kBulkWarps * 32) bulk_move_kernel(const MoveDev a) {
  extern __shared__ __align__(128) char bulk_smem[];
  __shared__ __align__(8) uint64_t bars[kBulkWarps][2];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  char* bank[2] = {bulk_smem + (size_t)(2 * warp) * kBulkBank, bulk_smem + (size_t)(2 * warp + 1) * kBulkBank};
  const uint32_t bar[2] = {smem_addr(&bars[warp][0]), smem_addr(&bars[warp][1])};
  if (lane == 0) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar[0]));
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar[1]));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncwarp();
  const int64_t row = a.row_bytes;
  const int rows = a.rows_per_cta;                    // rows per tile (<= 32)
  const char* sk = a.src.base_k;
  const char* sv = a.src.base_v;
  char* dk = const_cast<char*>(a.dst.base_k);
  char* dv = const_cast<char*>(a.dst.base_v);
  const int nw = gridDim.x * kBulkWarps;

  // The rows of tile w in the lanes; n = 0 for a tile past its segment's count.
  auto resolve = [&](int w) {
    BulkTile t{-1, -1, 0};
    const int seg = w / a.tiles;
    const int tile = w - seg * a.tiles;
    const int b = seg / a.heads;
    const int h = seg - b * a.heads;
    int count = a.rows_max;
    if (a.counts) {
      count = a.counts[(int64_t)b * a.cnt_sb + (int64_t)h * a.cnt_sh];
      if (count > a.rows_max) count = a.rows_max;
    }
    const int r0 = tile * rows;
    if (r0 >= count) return t;
    t.n = min(rows, count - r0);
    if (lane < t.n) {
      const int i = r0 + lane;
      uint32_t why = 0;
      int64_t st;
      if (a.idx) {
        const int64_t o = (int64_t)b * a.idx_sb + (int64_t)h * a.idx_sh + i;
        st = a.idx64 ? static_cast<const int64_t*>(a.idx)[o] : (int64_t) static_cast<const int32_t*>(a.idx)[o];
      } else {
        st = (a.src.tok0 ? a.src.tok0[b] : 0) + (int64_t)i;
      }
      const int64_t dt = (a.dst.tok0 ? a.dst.tok0[b] : 0) + (int64_t)i;
      t.so = rows_offset(a.src, b, h, st, &why, MSKV_STATUS_INDEX_OOB);
      t.dof = rows_offset(a.dst, b, h, dt, &why, MSKV_STATUS_DST_OOB);
      if (why && a.status) atomicOr(a.status, why);
    }
    return t;
  };
  // The next non-empty tile of this warp at or after w (w >= work: none).
  auto next = [&](int& w, BulkTile& t) {
    while (w < a.work) {
      t = resolve(w);
      if (t.n) return;
      w += nw;
    }
  };
  // Rows of tile t into bank k: zero-filled destination rows for invalid sources (the lanes'
  // own stores), one bulk copy per valid row (lane 0), the bank's expected bytes on its barrier.
  auto issue = [&](const BulkTile& t, int k) {
    uint32_t bytes = 0;
    for (int i = 0; i < t.n; ++i) {
      const int64_t so = __shfl_sync(0xffffffffu, t.so, i);
      const int64_t dof = __shfl_sync(0xffffffffu, t.dof, i);
      if (dof < 0) continue;
      if (so < 0) {
        if (a.zero_invalid)
          for (int64_t c = lane; c < row / 16; c += 32) {
            reinterpret_cast<uint4*>(dk + dof)[c] = make_uint4(0, 0, 0, 0);
            if (HAS_V) reinterpret_cast<uint4*>(dv + dof)[c] = make_uint4(0, 0, 0, 0);
          }
        continue;
      }
      bytes += (uint32_t)row * (HAS_V ? 2 : 1);
    }
    if (lane == 0) {
      asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar[k]), "r"(bytes) : "memory");
    }
    for (int i = 0; i < t.n; ++i) {
      const int64_t so = __shfl_sync(0xffffffffu, t.so, i);
      const int64_t dof = __shfl_sync(0xffffffffu, t.dof, i);
      if (lane == 0 && so >= 0 && dof >= 0) {
        bulk_load(smem_addr(bank[k] + (size_t)i * row), sk + so, (uint32_t)row, bar[k]);
        if (HAS_V) bulk_load(smem_addr(bank[k] + (size_t)(rows + i) * row), sv + so, (uint32_t)row, bar[k]);
      }
    }
  };
  auto drain = [&](const BulkTile& t, int k) {
    for (int i = 0; i < t.n; ++i) {
      const int64_t so = __shfl_sync(0xffffffffu, t.so, i);
      const int64_t dof = __shfl_sync(0xffffffffu, t.dof, i);
      if (lane == 0 && so >= 0 && dof >= 0) {
        bulk_store(dk + dof, smem_addr(bank[k] + (size_t)i * row), (uint32_t)row);
        if (HAS_V) bulk_store(dv + dof, smem_addr(bank[k] + (size_t)(rows + i) * row), (uint32_t)row);
      }
    }
    if (lane == 0) asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  };

  int w = blockIdx.x * kBulkWarps + warp;
  BulkTile cur{-1, -1, 0}, nxt{-1, -1, 0};
  next(w, cur);
  uint32_t phase[2] = {0, 0};
  int k = 0;
  if (w < a.work) issue(cur, 0);
  bool pending_other = false;                         // the other bank has copies in flight
  while (w < a.work) {
    int wn = w + nw;
    next(wn, nxt);
    if (wn < a.work) {
      // bank k^1 was last drained two tiles ago: its stores must have read it
      if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
      __syncwarp();
      issue(nxt, k ^ 1);
      pending_other = true;
    }
    uint32_t ok = 0;
    if (lane == 0) ok = bulk_wait(bar[k], phase[k]);
    ok = __shfl_sync(0xffffffffu, ok, 0);
    if (!ok) {                                        // give up: record it, let the rest land
      if (lane == 0) {
        if (a.status) atomicOr(a.status, MSKV_STATUS_TIMEOUT);
        if (pending_other) bulk_wait(bar[k ^ 1], phase[k ^ 1]);
        asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      }
      return;
    }
    phase[k] ^= 1;
    drain(cur, k);
    pending_other = false;
    w = wn;
    cur = nxt;
    k ^= 1;
  }
  if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// Largest power-of-two vector width (<= 16 bytes) that divides the row size, every stride
// and every base pointer of both sides.
static int pick_vec(const MoveDev& m) {
  uint64_t bits = (uint64_t)m.row_bytes;
  auto add = [&](uint64_t v) { bits |= v; };
  for (const RowsDev* r : {&m.src, &m.dst}) {
    add((uint64_t)(uintptr_t)r->base_k);
    if (r->base_v) add((uint64_t)(uintptr_t)r->base_v);
    if (r->page_table) {
      add((uint64_t)r->sp); add((uint64_t)r->sh); add((uint64_t)r->st);
    } else {
      add((uint64_t)r->sb); add((uint64_t)r->sh); add((uint64_t)r->st);
    }
  }
  for (int v = 16; v > 1; v >>= 1)
    if ((bits & (uint64_t)(v - 1)) == 0) return v;
  return 1;
}

// CTAs of a move that reads or writes host memory.  Every row load a CTA issues stays in
// flight for the PCIe round trip, and loads queued behind the host link also hold up the HBM
// traffic of kernels running beside the move.  The link needs only bandwidth x latency in
// flight (tens to hundreds of KB), so a bounded grid (about 32 KB per CTA per round) keeps it
// busy without flooding the memory system; HBM-only moves use the full grid.
constexpr int kHostLinkCtas = 32;

static int launch_move(MoveDev m, cudaStream_t stream, const char* what, int max_ctas, bool host) {
  const int64_t segs = (int64_t)m.batch * m.heads;
  if (segs == 0 || m.rows_max == 0) return MSKV_OK;
  const int vec = pick_vec(m);
  const bool has_v = m.src.base_v != nullptr && m.dst.base_v != nullptr;
  if (host && vec == 16 && m.row_bytes >= kBulkMinRow && m.row_bytes <= (has_v ? kBulkMaxRow : kBulkBank)) {
    // bulk copies: tiles of up to 32 rows per warp, two banks per warp
    int rows = (int)(kBulkBank / (m.row_bytes * (has_v ? 2 : 1)));
    rows = rows > 32 ? 32 : rows;
    if (rows > m.rows_max) rows = m.rows_max;
    m.rows_per_cta = rows;
    m.tiles = (m.rows_max + rows - 1) / rows;
    const int64_t work = segs * m.tiles;
    if (work > 0x7fffffffLL) return fail(MSKV_ERR_RANGE, "%s: grid too large", what);
    m.work = (int)work;
    int64_t blocks = (work + kBulkWarps - 1) / kBulkWarps;      // one tile per warp at most
    if (max_ctas > 0 && max_ctas < blocks) blocks = max_ctas;
    const int smem = 2 * kBulkWarps * kBulkBank;
    const void* kern = has_v ? (const void*)bulk_move_kernel<true> : (const void*)bulk_move_kernel<false>;
    int rc = ensure_smem_limit(kern, smem, what);
    if (rc) return rc;
    if (has_v) bulk_move_kernel<true><<<(unsigned)blocks, kBulkWarps * 32, smem, stream>>>(m);
    else bulk_move_kernel<false><<<(unsigned)blocks, kBulkWarps * 32, smem, stream>>>(m);
    return after_launch(what);
  }
  const int64_t chunks = m.row_bytes / vec;
  int rows = (int)(((int64_t)kThreads * kUnroll) / (chunks > 0 ? chunks : 1));
  rows = rows < 1 ? 1 : (rows > kMaxRowsPerCta ? kMaxRowsPerCta : rows);
  if (rows > m.rows_max) rows = m.rows_max;
  m.rows_per_cta = rows;
  m.tiles = (m.rows_max + rows - 1) / rows;
  m.chunk_shift = -1;
  if ((chunks & (chunks - 1)) == 0) {
    int s = 0;
    while ((1LL << s) < chunks) ++s;
    m.chunk_shift = s;
  }
  const int64_t work = segs * m.tiles;
  if (work > 0x7fffffffLL) return fail(MSKV_ERR_RANGE, "%s: grid too large", what);
  m.work = (int)work;
  const int64_t blocks = max_ctas > 0 && max_ctas < work ? max_ctas : work;
  switch (vec) {
    case 16: move_rows_kernel<16><<<(unsigned)blocks, kThreads, 0, stream>>>(m); break;
    case 8: move_rows_kernel<8><<<(unsigned)blocks, kThreads, 0, stream>>>(m); break;
    case 4: move_rows_kernel<4><<<(unsigned)blocks, kThreads, 0, stream>>>(m); break;
    case 2: move_rows_kernel<2><<<(unsigned)blocks, kThreads, 0, stream>>>(m); break;
    default: move_rows_kernel<1><<<(unsigned)blocks, kThreads, 0, stream>>>(m); break;
  }
  return after_launch(what);
}

// Resolves the device-accessible address of a (possibly host) base pointer; *host is set
// when the memory lives on the host side of the link.
static int resolve(const void* p, const void** out, const char* what, bool* host = nullptr) {
  if (!p) { *out = nullptr; return MSKV_OK; }
  void* d = nullptr;
  int rc = mskv_device_view(p, &d);
  if (rc != MSKV_OK) return fail(rc, "%s: %s", what, mskv_last_error());
  if (host && d != p) *host = true;
  if (host && d == p) {
    cudaPointerAttributes at;
    if (cudaPointerGetAttributes(&at, p) == cudaSuccess && at.type == cudaMemoryTypeHost) *host = true;
    cudaGetLastError();
  }
  *out = d;
  return MSKV_OK;
}

static int resolve_rows(mskv_rows& r, const char* side, bool* host) {
  int rc = resolve(r.base_k, &r.base_k, side, host);
  if (rc) return rc;
  return resolve(r.base_v, &r.base_v, side, host);
}

static int grid_cap(int requested, bool host) {
  if (requested > 0) return requested;
  return host ? kHostLinkCtas : 0;
}

}  // namespace mskv

using namespace mskv;

extern "C" {

int mskv_uva_gather(const void* k_in, const void* v_in, const int64_t* indices,
                    int64_t num_selected, int64_t batch_size, int64_t num_heads,
                    int64_t seq_len, int64_t head_dim, int32_t elem_bytes,
                    void* k_out, void* v_out, uint32_t* status, void* stream) {
  if (!k_in || !v_in || !k_out || !v_out) return fail(MSKV_ERR_ARG, "mskv_uva_gather: NULL tensor pointer");
  if (num_selected < 0 || batch_size < 0 || num_heads < 0 || seq_len < 0 || head_dim < 0)
    return fail(MSKV_ERR_ARG, "mskv_uva_gather: negative size");
  if (elem_bytes != 1 && elem_bytes != 2 && elem_bytes != 4 && elem_bytes != 8)
    return fail(MSKV_ERR_DTYPE, "mskv_uva_gather: unsupported element size %d", elem_bytes);
  if (num_selected > 0x7fffffffLL || batch_size > 0x7fffffffLL || num_heads > 0x7fffffffLL ||
      batch_size * num_heads > 0x7fffffffLL)
    return fail(MSKV_ERR_RANGE, "mskv_uva_gather: size exceeds int32");
  if (num_selected > 0 && !indices) return fail(MSKV_ERR_ARG, "mskv_uva_gather: indices is NULL");
  if (num_selected == 0 || batch_size == 0 || num_heads == 0 || head_dim == 0) return MSKV_OK;
  const int64_t row = head_dim * elem_bytes;
  mskv_rows src{};
  src.base_k = k_in; src.base_v = v_in;
  src.stride_t = row; src.stride_h = seq_len * row; src.stride_b = num_heads * seq_len * row;
  src.len_scalar = seq_len;
  mskv_rows dst{};
  dst.base_k = k_out; dst.base_v = v_out;
  dst.stride_t = row; dst.stride_h = num_selected * row; dst.stride_b = num_heads * num_selected * row;
  dst.len_scalar = num_selected;
  bool host = false;
  int rc = resolve_rows(src, "mskv_uva_gather k_in/v_in", &host);
  if (rc) return rc;
  rc = resolve_rows(dst, "mskv_uva_gather k_out/v_out", &host);
  if (rc) return rc;
  const void* idx_dev = nullptr;
  rc = resolve(indices, &idx_dev, "mskv_uva_gather indices");
  if (rc) return rc;
  MoveDev m{};
  m.src = to_dev(src); m.dst = to_dev(dst);
  m.idx = idx_dev; m.idx64 = 1; m.idx_sb = 0; m.idx_sh = 0;
  m.row_bytes = row; m.status = status; m.batch = (int)batch_size; m.heads = (int)num_heads;
  m.rows_max = (int)num_selected; m.zero_invalid = 1;
  return launch_move(m, as_stream(stream), "mskv_uva_gather", grid_cap(0, host), host);
}

int mskv_gather(const mskv_gather_desc* d, void* stream) {
  if (!d) return fail(MSKV_ERR_ARG, "mskv_gather: NULL descriptor");
  if (d->batch < 0 || d->heads < 0 || d->num_selected < 0 || d->row_bytes <= 0)
    return fail(MSKV_ERR_ARG, "mskv_gather: bad sizes");
  if (d->index_bits != 32 && d->index_bits != 64) return fail(MSKV_ERR_ARG, "mskv_gather: index_bits must be 32 or 64");
  if ((int64_t)d->batch * d->heads == 0 || d->num_selected == 0) return MSKV_OK;
  if (!d->indices) return fail(MSKV_ERR_ARG, "mskv_gather: indices is NULL");
  mskv_rows src = d->src, dst = d->dst;
  const bool need_v = src.base_v != nullptr || dst.base_v != nullptr;
  int rc = check_rows(src, "mskv_gather src", need_v);
  if (rc) return rc;
  rc = check_rows(dst, "mskv_gather dst", need_v);
  if (rc) return rc;
  if (d->max_ctas < 0) return fail(MSKV_ERR_ARG, "mskv_gather: negative max_ctas");
  bool host = false;
  if ((rc = resolve_rows(src, "mskv_gather src", &host))) return rc;
  if ((rc = resolve_rows(dst, "mskv_gather dst", &host))) return rc;
  MoveDev m{};
  m.src = to_dev(src); m.dst = to_dev(dst);
  m.idx = d->indices; m.idx64 = d->index_bits == 64; m.idx_sb = d->idx_stride_b; m.idx_sh = d->idx_stride_h;
  m.counts = d->counts; m.cnt_sb = d->cnt_stride_b; m.cnt_sh = d->cnt_stride_h;
  m.row_bytes = d->row_bytes; m.status = d->status; m.batch = d->batch; m.heads = d->heads;
  m.rows_max = d->num_selected; m.zero_invalid = 1;
  return launch_move(m, as_stream(stream), "mskv_gather", grid_cap(d->max_ctas, host), host);
}

int mskv_copy_rows(const mskv_copy_desc* d, void* stream) {
  if (!d) return fail(MSKV_ERR_ARG, "mskv_copy_rows: NULL descriptor");
  if (d->batch < 0 || d->heads < 0 || d->num_tokens < 0 || d->row_bytes <= 0)
    return fail(MSKV_ERR_ARG, "mskv_copy_rows: bad sizes");
  if ((int64_t)d->batch * d->heads == 0 || d->num_tokens == 0) return MSKV_OK;
  mskv_rows src = d->src, dst = d->dst;
  const bool need_v = src.base_v != nullptr || dst.base_v != nullptr;
  int rc = check_rows(src, "mskv_copy_rows src", need_v);
  if (rc) return rc;
  rc = check_rows(dst, "mskv_copy_rows dst", need_v);
  if (rc) return rc;
  if (d->max_ctas < 0) return fail(MSKV_ERR_ARG, "mskv_copy_rows: negative max_ctas");
  bool host = false;
  if ((rc = resolve_rows(src, "mskv_copy_rows src", &host))) return rc;
  if ((rc = resolve_rows(dst, "mskv_copy_rows dst", &host))) return rc;
  MoveDev m{};
  m.src = to_dev(src); m.dst = to_dev(dst);
  m.idx = nullptr;
  m.counts = d->counts; m.cnt_sb = 1; m.cnt_sh = 0;
  m.row_bytes = d->row_bytes; m.status = d->status; m.batch = d->batch; m.heads = d->heads;
  m.rows_max = d->num_tokens; m.zero_invalid = 0;
  return launch_move(m, as_stream(stream), "mskv_copy_rows", grid_cap(d->max_ctas, host), host);
}

}  // extern "C"
