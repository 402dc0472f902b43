// Device-resident decode lane state: the per-step bookkeeping the host scheduler used to redo and
// upload before every decode step.
//
// A decode batch lives in static device buffers (ids / pos / slot / ctx / block table, one row per
// lane); the CUDA graph of a decode step ends with k_decode_advance, which turns this step's
// sampled tokens into the next step's inputs on the device:
//   ids[b] <- next[b];  pos[b] += 1;  ctx[b] = pos[b] + 1;  slot[b] <- page of pos[b] from the table.
// The host only appends block-table entries when a lane crosses into a page it has not mapped yet
// (k_scatter_i32, a few entries every 16 steps per lane) and reads the sampled tokens back one step
// behind, so it schedules step t + 1 while the GPU runs step t.  Padding lanes (slot < 0) stay idle.
//
// Reference: the host loop of NativeScheduler.run (internal/modelengine/nativesched.go:227), which
// rebuilds the step's inputs for BatchSession.StepBatch (internal/model/batch_step.go:7) on the host
// before every token.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "common.cuh"

using namespace fak;

namespace {

constexpr int kPage = 16;

__global__ void k_decode_advance(const int* __restrict__ next, int* __restrict__ ids, int* __restrict__ pos,
                                 int* __restrict__ slot, int* __restrict__ ctx, const int* __restrict__ bt,
                                 int bt_stride, int B) {
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B && slot[b] >= 0) {
    const int p = pos[b] + 1;
    const int pg = p / kPage;
    ids[b] = next[b];
    pos[b] = p;
    ctx[b] = p + 1;
    // a position past the table (the lane cannot run again) maps to no slot: no KV write
    slot[b] = pg < bt_stride ? bt[(int64_t)b * bt_stride + pg] * kPage + (p % kPage) : -1;
  }
  pdl_launch_dependents();
}

__global__ void k_scatter_i32(int* __restrict__ dst, const int* __restrict__ idx_val, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) dst[idx_val[2 * i]] = idx_val[2 * i + 1];
}

}  // namespace

// next [>=B] int32 (this step's sampled tokens); ids/pos/slot/ctx [>=B] int32; bt [>=B, W] int32.
void decode_advance(torch::Tensor next, torch::Tensor ids, torch::Tensor pos, torch::Tensor slot, torch::Tensor ctx,
                    torch::Tensor bt, int64_t B) {
  for (auto* t : {&next, &ids, &pos, &slot, &ctx})
    TORCH_CHECK(t->is_cuda() && t->scalar_type() == torch::kInt32 && t->is_contiguous() && t->numel() >= B,
                "decode_advance: int32 [>=B] device vectors");
  TORCH_CHECK(bt.scalar_type() == torch::kInt32 && bt.dim() == 2 && bt.stride(1) == 1 && bt.size(0) >= B,
              "decode_advance: block table [>=B, W] int32");
  if (B <= 0) return;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)((B + 127) / 128));
  cfg.blockDim = dim3(128);
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_decode_advance, (const int*)next.data_ptr<int>(), ids.data_ptr<int>(),
                                    pos.data_ptr<int>(), slot.data_ptr<int>(), ctx.data_ptr<int>(),
                                    (const int*)bt.data_ptr<int>(), (int)bt.stride(0), (int)B));
}

// dst.flatten()[idx_val[2i]] = idx_val[2i + 1] for i < n (idx_val int32 [n, 2] on the device).
void scatter_i32(torch::Tensor dst, torch::Tensor idx_val, int64_t n) {
  TORCH_CHECK(dst.is_cuda() && dst.scalar_type() == torch::kInt32 && dst.is_contiguous(), "scatter_i32: dst");
  TORCH_CHECK(idx_val.is_cuda() && idx_val.scalar_type() == torch::kInt32 && idx_val.is_contiguous() &&
                  idx_val.numel() >= 2 * n, "scatter_i32: idx_val [n, 2] int32");
  if (n <= 0) return;
  k_scatter_i32<<<(unsigned)((n + 127) / 128), 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      dst.data_ptr<int>(), (const int*)idx_val.data_ptr<int>(), (int)n);
  FAK_CUDA_CHECK(cudaGetLastError());
}
