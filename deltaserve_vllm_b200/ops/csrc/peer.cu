// Peer-mapped workspaces for the fused compute + collective kernels.
//
// Each rank allocates one block with cudaMalloc (outside PyTorch's caching
// allocator, so the whole block is one IPC-exportable allocation), zeroes it,
// and exports a CUDA IPC handle. The handles travel over the host process
// group; every rank opens the others' blocks (plain P2P mappings over NVLink,
// no multicast object), so a kernel can load from and store to any rank's
// block with ordinary global-memory instructions.
#include <torch/extension.h>
#include <c10/cuda/CUDAException.h>
#include <cuda_runtime.h>

#include <cstring>
#include <string>

// Allocate `bytes` on the current device, zeroed; returns (address, ipc handle bytes).
std::tuple<int64_t, std::string> dsv_peer_alloc(int64_t bytes) {
  TORCH_CHECK(bytes > 0, "dsv_peer_alloc: size must be positive");
  void* p = nullptr;
  C10_CUDA_CHECK(cudaMalloc(&p, (size_t)bytes));
  C10_CUDA_CHECK(cudaMemset(p, 0, (size_t)bytes));
  C10_CUDA_CHECK(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  C10_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  return {reinterpret_cast<int64_t>(p), std::string(reinterpret_cast<const char*>(&h), sizeof(h))};
}

// Map another rank's block into this process; returns its address here.
int64_t dsv_peer_open(const std::string& handle) {
  TORCH_CHECK(handle.size() == sizeof(cudaIpcMemHandle_t), "dsv_peer_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  C10_CUDA_CHECK(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
  return reinterpret_cast<int64_t>(p);
}

void dsv_peer_close(int64_t addr) {
  C10_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(addr)));
}

void dsv_peer_free(int64_t addr) { C10_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(addr))); }

// Zero a range of this rank's own block (flags after an aborted run).
void dsv_peer_zero(int64_t addr, int64_t bytes) {
  C10_CUDA_CHECK(cudaMemset(reinterpret_cast<void*>(addr), 0, (size_t)bytes));
}

// A tensor over `addr` on `device` (memory owned by a peer workspace block,
// never freed through PyTorch).
torch::Tensor dsv_peer_view(int64_t addr, std::vector<int64_t> shape, c10::ScalarType dtype, int64_t device) {
  auto opts = torch::TensorOptions().dtype(dtype).device(torch::kCUDA, (int)device);
  return torch::from_blob(reinterpret_cast<void*>(addr), shape, opts);
}
