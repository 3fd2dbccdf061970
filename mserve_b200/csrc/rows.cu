// Row movers: the selected-row gather from pinned host memory into HBM (mskv_uva_gather,
// mskv_gather) and the contiguous row copies behind the paged append and the host write-back
// (mskv_copy_rows).
//
// Design (B200): the work is tiles of rows of one (b, h) segment; a CTA takes tiles in a
// grid-stride loop (a bounded grid for moves that touch host memory, see launch_move).  For
// each tile the first threads resolve the source/destination byte offsets (index list, ring,
// page table, bounds) into shared memory once per row; then all 256 threads stream the tile
// as VEC-byte chunks with UNROLL independent loads in flight per thread for K and for V
// before any store.
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

template <int VEC>
__global__ void __launch_bounds__(kThreads) move_rows_kernel(const MoveDev a) {
  using V = typename Vec<VEC>::T;
  __shared__ int64_t s_src[kMaxRowsPerCta];
  __shared__ int64_t s_dst[kMaxRowsPerCta];

  const int64_t chunks = a.row_bytes / VEC;
  const char* __restrict__ sk = a.src.base_k;
  const char* __restrict__ sv = a.src.base_v;
  char* __restrict__ dk = const_cast<char*>(a.dst.base_k);
  char* __restrict__ dv = const_cast<char*>(a.dst.base_v);
  const bool has_v = sv != nullptr;

  // Grid-stride loop over the tiles: the grid may be smaller than the work (see launch_move).
  for (int w = blockIdx.x; w < a.work; w += gridDim.x) {
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
    if (r0 >= count) continue;  // uniform across the CTA
    const int nrows = min(a.rows_per_cta, count - r0);

    __syncthreads();  // the previous tile's readers of s_src / s_dst are done
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
    __syncthreads();

    const int64_t total = (int64_t)nrows * chunks;
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
          const int64_t so = s_src[r];
          const int64_t dof = s_dst[r];
          if (dof >= 0 && (so >= 0 || a.zero_invalid)) {
            dofs[u] = dof + c * VEC;
            if (so >= 0) {
              rk[u] = *reinterpret_cast<const V*>(sk + so + c * VEC);
              if (has_v) rv[u] = *reinterpret_cast<const V*>(sv + so + c * VEC);
            }
          }
        }
      }
#pragma unroll
      for (int u = 0; u < kUnroll; ++u) {
        if (dofs[u] >= 0) {
          *reinterpret_cast<V*>(dk + dofs[u]) = rk[u];
          if (has_v) *reinterpret_cast<V*>(dv + dofs[u]) = rv[u];
        }
      }
    }
  }
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

static int launch_move(MoveDev m, cudaStream_t stream, const char* what, int max_ctas) {
  const int64_t segs = (int64_t)m.batch * m.heads;
  if (segs == 0 || m.rows_max == 0) return MSKV_OK;
  const int vec = pick_vec(m);
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
  return launch_move(m, as_stream(stream), "mskv_uva_gather", grid_cap(0, host));
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
  return launch_move(m, as_stream(stream), "mskv_gather", grid_cap(d->max_ctas, host));
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
  return launch_move(m, as_stream(stream), "mskv_copy_rows", grid_cap(d->max_ctas, host));
}

}  // extern "C"
