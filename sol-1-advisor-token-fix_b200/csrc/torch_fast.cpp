// torch_fast.cpp — host binding for PyTorch callers of the full call.
//
// The same work as the Python fast path of attn_bwd_b200.attn_bwd (input checks,
// output allocation, the caller's current stream, the C-ABI call), done in C++ so a
// call costs a few microseconds of host time instead of ~12.  It calls the C-ABI
// entry point attn_bwd_b200 (include/attn_bwd_b200.h) and nothing else; the kernels
// live in libattn_bwd_b200.so.
//
// fast(dO, P, Pd, V, M, p) returns
//   (dS, dV)  on success,
//   an int    (the library's error code) when the call was made and failed,
//   None      when the inputs need the general path (other dtypes / shapes / strides /
//             devices, misaligned pointers): the Python side then converts and calls
//             the library through ctypes.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <c10/cuda/CUDAFunctions.h>
#include <c10/cuda/CUDAGuard.h>

#include "../../include/attn_bwd_b200.h"

namespace {

constexpr int64_t kHeads = 80, kKvHeads = 8, kHeadDim = 128;

inline bool dense16(const at::Tensor& t) {
  return t.is_contiguous() && (reinterpret_cast<uintptr_t>(t.data_ptr()) & 15u) == 0;
}

py::object fast(const at::Tensor& dO, const at::Tensor& P, const at::Tensor& Pd, const at::Tensor& V,
                const at::Tensor& M, double p) {
  if (!dO.is_cuda() || dO.scalar_type() != at::kBFloat16 || P.scalar_type() != at::kBFloat16 ||
      Pd.scalar_type() != at::kBFloat16 || V.scalar_type() != at::kBFloat16 || M.scalar_type() != at::kBool)
    return py::none();
  if (dO.dim() != 4 || V.dim() != 4 || P.dim() != 4 || Pd.dim() != 4 || M.dim() != 4) return py::none();
  const int64_t bs = dO.size(0), sq = dO.size(1), skv = V.size(2);
  if (dO.size(2) != kHeads || dO.size(3) != kHeadDim) return py::none();
  if (V.size(0) != bs || V.size(1) != kKvHeads || V.size(3) != kHeadDim) return py::none();
  const at::IntArrayRef ps = P.sizes();
  if (ps[0] != bs || ps[1] != kHeads || ps[2] != sq || ps[3] != skv || Pd.sizes() != ps || M.sizes() != ps)
    return py::none();
  const c10::Device dev = dO.device();
  if (P.device() != dev || Pd.device() != dev || V.device() != dev || M.device() != dev) return py::none();
  if (!dense16(dO) || !dense16(P) || !dense16(Pd) || !dense16(V) || !dense16(M)) return py::none();
  if (bs > INT32_MAX || sq > INT32_MAX || skv > INT32_MAX) return py::none();

  c10::cuda::OptionalCUDAGuard guard;
  if (dev.index() != c10::cuda::current_device()) guard.set_device(dev);
  at::Tensor dS = at::empty_like(P);
  at::Tensor dV = at::empty_like(V);
  const cudaStream_t stream = c10::cuda::getCurrentCUDAStream(dev.index()).stream();
  const int rc = attn_bwd_b200(dO.data_ptr(), P.data_ptr(), Pd.data_ptr(), V.data_ptr(),
                               static_cast<const uint8_t*>(M.data_ptr()), static_cast<float>(p), int(bs), int(sq),
                               int(skv), dS.data_ptr(), dV.data_ptr(), reinterpret_cast<attn_bwd_stream_t>(stream));
  if (rc != 0) return py::int_(rc);
  return py::make_tuple(dS, dV);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "C++ host binding of the attn_bwd_b200 full call for PyTorch tensors";
  m.def("fast", &fast, "full call on ready inputs: (dS, dV), an error code, or None");
}
