// Symmetric-heap back end without multicast: one cudaMalloc'd heap per rank, shared with the other
// ranks of the node through CUDA IPC handles (plain NVLink peer mappings).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>

#include "check.h"

#include <cstring>

namespace {

void ok(cudaError_t e, const char* what) { COB_CHECK(e == cudaSuccess, what, ": ", cudaGetErrorString(e)); }

// Device allocation owned by the returned uint8 tensor (freed with cudaFree when it dies).
torch::Tensor ipc_alloc(int64_t bytes, int64_t device) {
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  ok(cudaMalloc(&p, (size_t)bytes), "cudaMalloc (symmetric heap)");
  ok(cudaMemset(p, 0, (size_t)bytes), "cudaMemset");
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, (c10::DeviceIndex)device);
  return torch::from_blob(p, {bytes}, [](void* q) { cudaFree(q); }, opts);
}

pybind11::bytes ipc_handle(torch::Tensor heap) {
  const c10::cuda::CUDAGuard g(heap.device());
  cudaIpcMemHandle_t h;
  ok(cudaIpcGetMemHandle(&h, heap.data_ptr()), "cudaIpcGetMemHandle");
  return pybind11::bytes(reinterpret_cast<const char*>(&h), sizeof(h));
}

int64_t ipc_open(pybind11::bytes handle, int64_t device) {
  const std::string s = handle;
  COB_CHECK(s.size() == sizeof(cudaIpcMemHandle_t), "bad IPC handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, s.data(), sizeof(h));
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  void* p = nullptr;
  ok(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr, int64_t device) {
  const c10::cuda::CUDAGuard g((c10::DeviceIndex)device);
  ok(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr)), "cudaIpcCloseMemHandle");
}

}  // namespace

void register_ipc(pybind11::module& m) {
  m.def("ipc_alloc", &ipc_alloc);
  m.def("ipc_handle", &ipc_handle);
  m.def("ipc_open", &ipc_open);
  m.def("ipc_close", &ipc_close);
}
