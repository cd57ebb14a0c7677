// rowstream.cu -- host side of the row-stream GEMV: launch geometry and dispatch over the
// weight formats.  The kernel template is in rowstream_kernel.cuh; the Q8_0 and Q4_K formats are
// instantiated here, the other GGUF types in rowstream_more.cu.
#include "rowstream_kernel.cuh"

namespace ex {

int rowstream_max_m(Fmt fmt, int K, const DeviceInfo& dev) {
  (void)dev;
  const int per = act_bytes_total(fmt, K, 1) + 64;
  const int m = per > ACT_BUDGET ? 0 : ACT_BUDGET / per;
  return m < MAX_M ? m : MAX_M;
}

bool rowstream_quantizes_itself(Fmt fmt, int m) { return act_of(fmt) != Act::F32 && m <= PROLOGUE_QUANT_MAX_M; }

cudaError_t launch_rowstream(const RowStreamArgs& in, const DeviceInfo& dev, cudaStream_t st) {
  RowStreamArgs a = in;
  if (a.n_seg <= 0) {  // one tensor: it is segment 0
    a.n_seg = 1;
    a.seg[0] = RowSeg{a.w, a.n_rows, a.bias, a.out, 0};
  } else {
    if (a.n_seg > MAX_SEGS || a.mode != RowOut::Store) return cudaErrorInvalidValue;
    a.n_rows = 0;
    for (int i = 0; i < a.n_seg; ++i) a.n_rows += a.seg[i].n_rows;
  }
  if (a.mode == RowOut::StoreTp && (a.tp.world < 2 || a.tp.world > TP_MAX_WORLD ||
                                    (a.fmt != Fmt::Q8_0xQ8_0 && a.fmt != Fmt::Q4_KxQ8_K)))
    return cudaErrorInvalidValue;
  if (a.n_rows <= 0 || a.m <= 0) return cudaSuccess;
  if (a.m > MAX_M || a.K % (act_of(a.fmt) == Act::Q8_0 ? QK8_0 : QK_K) != 0) return cudaErrorInvalidValue;
  Layout L{};
  L.stage_bytes = STAGE_TARGET;
  if (a.row_bytes + STAGE_SLACK > L.stage_bytes) L.stage_bytes = (a.row_bytes + STAGE_SLACK + 127) & ~127;
  const bool exact = a.exact && (a.mode == RowOut::Store || a.mode == RowOut::Argmax);
  const int act = (act_bytes_total(a.fmt, a.K, a.m) + 127) & ~127;
  L.row_stride = a.row_bytes;
  if (exact) {
    // The EX_ROWS rows of a warp pass are read at the same offsets at once: rows whose length is a
    // multiple of 128 bytes would all fall in the same shared-memory banks.  Rows of 16-byte multiples
    // are copied one by one into slots of stride = 32 (mod 128) bytes, which spreads a pass over all
    // banks; other lengths are already staggered.
    if (a.row_bytes % 16 == 0) L.row_stride = a.row_bytes + ((32 - a.row_bytes % 128) + 128) % 128;
    // A warp owns its rows for a whole row's chain: stages of exactly EX_ROWS rows (where 3 fit) keep
    // as many warp passes in flight as shared memory allows.
    const int want = (EX_ROWS * L.row_stride + STAGE_SLACK + 127) & ~127;
    if (3 * want <= dev.max_smem_optin - BAR_BYTES - act) {
      L.stage_bytes = want;
    } else {
      L.row_stride = a.row_bytes;
    }
  }
  const int r_cap = (L.stage_bytes - STAGE_SLACK) / L.row_stride;
  long long r_want = (a.n_rows + 3LL * dev.sm_count - 1) / (3LL * dev.sm_count);
  if (r_want < 1) r_want = 1;
  if (exact) {  // tiles of whole warp passes
    r_want = (r_want + EX_ROWS - 1) / EX_ROWS * EX_ROWS;
    const int cap8 = r_cap / EX_ROWS * EX_ROWS;
    L.tile_rows = static_cast<int>(cap8 == 0 ? r_cap : (r_want < cap8 ? r_want : cap8));
  } else {
    L.tile_rows = static_cast<int>(r_want < r_cap ? r_want : r_cap);
  }
  L.n_tiles = 0;
  for (int i = 0; i < a.n_seg; ++i) {  // tiles never straddle two tensors
    a.seg[i].tile0 = L.n_tiles;
    L.n_tiles += (a.seg[i].n_rows + L.tile_rows - 1) / L.tile_rows;
  }
  L.act_off = BAR_BYTES;
  L.part_off = L.act_off + act;
  const int part = rowstream_sliced(a) ? (MAX_STAGES * L.tile_rows * (SLICE_UNITS * 4 + 4) + 127) & ~127 : 0;
  L.stage_off = L.part_off + part;
  int S = (dev.max_smem_optin - L.stage_off) / L.stage_bytes;
  if (S > MAX_STAGES) S = MAX_STAGES;
  if (S < 2) return cudaErrorInvalidConfiguration;
  L.n_stages = S;
  L.smem_total = L.stage_off + S * L.stage_bytes;
  const int grid = static_cast<int>(L.n_tiles < dev.sm_count ? L.n_tiles : dev.sm_count);

  switch (a.fmt) {
    case Fmt::Q8_0xQ8_0:
      if (a.mode == RowOut::Store) return launch_mtok<Fmt::Q8_0xQ8_0, RowOut::Store>(a, L, grid, st);
      if (a.mode == RowOut::StoreTp) return launch_mtok<Fmt::Q8_0xQ8_0, RowOut::StoreTp>(a, L, grid, st);
      if (a.mode == RowOut::Argmax) return launch_mtok<Fmt::Q8_0xQ8_0, RowOut::Argmax>(a, L, grid, st);
      return launch_mtok<Fmt::Q8_0xQ8_0, RowOut::Partials>(a, L, grid, st);
    case Fmt::Q4_KxQ8_K:
      if (a.mode == RowOut::Store) return launch_mtok<Fmt::Q4_KxQ8_K, RowOut::Store>(a, L, grid, st);
      if (a.mode == RowOut::StoreTp) return launch_mtok<Fmt::Q4_KxQ8_K, RowOut::StoreTp>(a, L, grid, st);
      if (a.mode == RowOut::Argmax) return launch_mtok<Fmt::Q4_KxQ8_K, RowOut::Argmax>(a, L, grid, st);
      return launch_mtok<Fmt::Q4_KxQ8_K, RowOut::Partials>(a, L, grid, st);
    case Fmt::Q4_KxF32:
      if (a.mode == RowOut::Store) return launch_mtok<Fmt::Q4_KxF32, RowOut::Store>(a, L, grid, st);
      if (a.mode == RowOut::Argmax) return launch_mtok<Fmt::Q4_KxF32, RowOut::Argmax>(a, L, grid, st);
      return cudaErrorInvalidValue;
    default:
      return launch_rowstream_more(a, L, grid, st);
  }
}

}  // namespace ex
