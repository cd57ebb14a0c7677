// rowstream_more.cu -- row-stream GEMV instantiations for the other GGUF weight types behind the
// same dispatch: Q4_0 and Q5_0 (Q8_0 activations), Q5_K and Q6_K (Q8_K activations, and fp32
// activations on the logits path).  Store, Argmax and Partials epilogues; the
// tensor-parallel epilogue is built for Q8_0 and Q4_K only (rowstream.cu).
#include "rowstream_kernel.cuh"

namespace ex {
namespace {

template <Fmt F>
cudaError_t launch_modes(const RowStreamArgs& a, const Layout& L, int grid, cudaStream_t st) {
  if constexpr (act_of(F) == Act::F32) {  // the logits path: one hidden state; argmax, or every score
    if (a.mode == RowOut::Argmax && a.m == 1)
      return a.exact ? launch_impl<F, RowOut::Argmax, 1, false, true>(a, L, grid, st)
                     : launch_impl<F, RowOut::Argmax, 1>(a, L, grid, st);
    if (a.mode == RowOut::Store && a.m == 1)
      return a.exact ? launch_impl<F, RowOut::Store, 1, false, true>(a, L, grid, st)
                     : launch_impl<F, RowOut::Store, 1>(a, L, grid, st);
  } else {
    if (a.mode == RowOut::Store) return launch_mtok<F, RowOut::Store>(a, L, grid, st);
    if (a.mode == RowOut::Argmax) return launch_mtok<F, RowOut::Argmax>(a, L, grid, st);
    if (a.mode == RowOut::Partials) return launch_mtok<F, RowOut::Partials>(a, L, grid, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_rowstream_more(const RowStreamArgs& a, const Layout& L, int grid, cudaStream_t st) {
  switch (a.fmt) {
    case Fmt::Q4_0xQ8_0: return launch_modes<Fmt::Q4_0xQ8_0>(a, L, grid, st);
    case Fmt::Q5_0xQ8_0: return launch_modes<Fmt::Q5_0xQ8_0>(a, L, grid, st);
    case Fmt::Q5_KxQ8_K: return launch_modes<Fmt::Q5_KxQ8_K>(a, L, grid, st);
    case Fmt::Q6_KxQ8_K: return launch_modes<Fmt::Q6_KxQ8_K>(a, L, grid, st);
    case Fmt::Q5_KxF32: return launch_modes<Fmt::Q5_KxF32>(a, L, grid, st);
    case Fmt::Q6_KxF32: return launch_modes<Fmt::Q6_KxF32>(a, L, grid, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace ex
