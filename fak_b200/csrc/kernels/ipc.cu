// Peer-mapped buffers for the in-kernel collectives, through CUDA IPC memory handles.
//
// Every rank allocates one plain device buffer (cudaMalloc, zeroed), exports its IPC handle, and
// opens every peer's handle (cudaIpcOpenMemHandle with lazy peer access): each rank's kernels then
// hold the device address of every peer's buffer and move data with ordinary loads and stores over
// NVLink/NVSwitch.  Unlike a multicast-capable symmetric allocation, nothing here is bound to an
// NVLink multicast object, so a rank that exits (or a test that makes a peer wait run out) leaves
// the other ranks' mappings plain peer mappings.  The handles travel between processes through the
// process group on the host (see parallel/p2p.py).
//
// Reference counterpart: the NCCL communicator set-up of internal/compute/cuda_nccl_pg.cu:54-72
// (ncclGetUniqueId / ncclCommInitRank), which this replaces for the fused collectives.
#include <torch/extension.h>

#include <cstring>

#include "common.cuh"

// Allocates nbytes on `device` (zero-filled) and returns {device pointer, IPC handle bytes}.
std::tuple<int64_t, torch::Tensor> ipc_alloc(int64_t nbytes, int64_t device) {
  TORCH_CHECK(nbytes > 0, "ipc_alloc: size");
  int prev = 0;
  FAK_CUDA_CHECK(cudaGetDevice(&prev));
  FAK_CUDA_CHECK(cudaSetDevice((int)device));
  void* p = nullptr;
  FAK_CUDA_CHECK(cudaMalloc(&p, (size_t)nbytes));
  FAK_CUDA_CHECK(cudaMemset(p, 0, (size_t)nbytes));
  FAK_CUDA_CHECK(cudaDeviceSynchronize());
  cudaIpcMemHandle_t h;
  FAK_CUDA_CHECK(cudaIpcGetMemHandle(&h, p));
  FAK_CUDA_CHECK(cudaSetDevice(prev));
  auto bytes = torch::empty({(int64_t)sizeof(h)}, torch::kUInt8);
  std::memcpy(bytes.data_ptr(), &h, sizeof(h));
  return {reinterpret_cast<int64_t>(p), bytes};
}

// Opens a peer's IPC handle on `device`; returns the peer buffer's address in this process.
int64_t ipc_open(torch::Tensor handle, int64_t device) {
  TORCH_CHECK(handle.scalar_type() == torch::kUInt8 && handle.numel() == (int64_t)sizeof(cudaIpcMemHandle_t),
              "ipc_open: handle bytes");
  auto h = handle.cpu().contiguous();
  cudaIpcMemHandle_t mh;
  std::memcpy(&mh, h.data_ptr(), sizeof(mh));
  int prev = 0;
  FAK_CUDA_CHECK(cudaGetDevice(&prev));
  FAK_CUDA_CHECK(cudaSetDevice((int)device));
  void* p = nullptr;
  FAK_CUDA_CHECK(cudaIpcOpenMemHandle(&p, mh, cudaIpcMemLazyEnablePeerAccess));
  FAK_CUDA_CHECK(cudaSetDevice(prev));
  return reinterpret_cast<int64_t>(p);
}

void ipc_close(int64_t ptr) { FAK_CUDA_CHECK(cudaIpcCloseMemHandle(reinterpret_cast<void*>(ptr))); }

void ipc_free(int64_t ptr) { FAK_CUDA_CHECK(cudaFree(reinterpret_cast<void*>(ptr))); }

// A uint8 tensor over [ptr, ptr + nbytes) of `device` (no ownership: ipc_free releases the memory).
torch::Tensor ipc_view(int64_t ptr, int64_t nbytes, int64_t device) {
  auto opts = torch::TensorOptions().dtype(torch::kUInt8).device(torch::kCUDA, (int)device);
  return torch::from_blob(reinterpret_cast<void*>(ptr), {nbytes}, opts);
}
