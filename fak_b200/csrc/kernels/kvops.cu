// KV-cache maintenance kernels.
//
// k_kv_move: moves token rows of the paged K/V cache ([L, P, Hkv, 16, D] bf16, all layers in one
// launch) from source slots to destination slots (slot = page * 16 + offset), re-rotating the keys
// of the rows flagged in `rot` back by a fixed number of positions n: a key stored as R(p) k
// becomes R(p - n) k = R(-n) R(p) k, with cos(n theta_j), sin(n theta_j) given per pair j (HF
// rotate_half pairing, j and j + D/2).  Values move unchanged.  This is how a span of positions
// is evicted from a sequence: the survivors after the span are renumbered down by its length, and
// the cache then holds what RoPE at the new positions gives (up to one bf16 rounding of the
// re-rotated keys).  Source and destination slots must not overlap (the caller writes into fresh
// pages).
//
// Grid (rows, layers); one thread per (kv head, pair).
// Reference: KVCache.Evict with re-RoPE renumbering (internal/model/kvcache.go:94-180), paged
// middle-span eviction (internal/model/paged_evict.go).
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "common.cuh"

namespace {

__global__ void k_kv_move(__nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, int64_t layer_stride,
                          int Hkv, int D, const int* __restrict__ src_slot, const int* __restrict__ dst_slot,
                          const uint8_t* __restrict__ rot, const float* __restrict__ cos_n,
                          const float* __restrict__ sin_n) {
  const int row = blockIdx.x, layer = blockIdx.y;
  const int half = D / 2;
  const int h = threadIdx.x / half, j = threadIdx.x % half;
  if (h >= Hkv) return;
  const int64_t ss = src_slot[row], ds = dst_slot[row];
  // slot s = page * 16 + offset -> element offset ((page * Hkv + h) * 16 + offset) * D
  const int64_t so = layer * layer_stride + (((ss >> 4) * Hkv + h) * 16 + (ss & 15)) * D;
  const int64_t d_o = layer * layer_stride + (((ds >> 4) * Hkv + h) * 16 + (ds & 15)) * D;
  const float x0 = __bfloat162float(kc[so + j]), x1 = __bfloat162float(kc[so + j + half]);
  float y0 = x0, y1 = x1;
  if (rot[row]) {
    const float c = cos_n[j], s = sin_n[j];
    y0 = x0 * c + x1 * s;   // rotate by -n: (x0, x1) -> (x0 c + x1 s, x1 c - x0 s)
    y1 = x1 * c - x0 * s;
  }
  kc[d_o + j] = __float2bfloat16_rn(y0);
  kc[d_o + j + half] = __float2bfloat16_rn(y1);
  vc[d_o + j] = vc[so + j];
  vc[d_o + j + half] = vc[so + j + half];
}

}  // namespace

void kv_move(torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor src_slot, torch::Tensor dst_slot,
             torch::Tensor rot, torch::Tensor cos_n, torch::Tensor sin_n) {
  TORCH_CHECK(k_cache.is_cuda() && k_cache.scalar_type() == torch::kBFloat16 && k_cache.dim() == 5 &&
                  k_cache.is_contiguous() && v_cache.sizes() == k_cache.sizes() && v_cache.is_contiguous(),
              "kv_move: caches [L, P, Hkv, 16, D] bf16");
  TORCH_CHECK(k_cache.size(3) == 16, "kv_move: page size 16");
  const int L = (int)k_cache.size(0), Hkv = (int)k_cache.size(2), D = (int)k_cache.size(4);
  const int64_t P = k_cache.size(1);
  const int T = (int)src_slot.numel();
  TORCH_CHECK(src_slot.scalar_type() == torch::kInt32 && dst_slot.scalar_type() == torch::kInt32 &&
                  dst_slot.numel() == T && rot.scalar_type() == torch::kUInt8 && rot.numel() == T,
              "kv_move: slots int32 [T], rot uint8 [T]");
  TORCH_CHECK(cos_n.scalar_type() == torch::kFloat32 && cos_n.numel() == D / 2 && sin_n.numel() == D / 2,
              "kv_move: cos/sin of the shift [D/2] f32");
  TORCH_CHECK(Hkv * D / 2 <= 1024, "kv_move: kv heads x head_dim / 2 must fit one block");
  if (T == 0) return;
  {  // slots in range (checked on the host copy the caller built)
    auto s = src_slot.cpu(), d = dst_slot.cpu();
    const int* sp = s.data_ptr<int>();
    const int* dp = d.data_ptr<int>();
    for (int i = 0; i < T; i++)
      TORCH_CHECK(sp[i] >= 0 && sp[i] < P * 16 && dp[i] >= 0 && dp[i] < P * 16, "kv_move: slot out of range");
  }
  auto stream = at::cuda::getCurrentCUDAStream();
  k_kv_move<<<dim3(T, L), Hkv * D / 2, 0, stream>>>(
      reinterpret_cast<__nv_bfloat16*>(k_cache.data_ptr()), reinterpret_cast<__nv_bfloat16*>(v_cache.data_ptr()),
      P * Hkv * 16 * D, Hkv, D, src_slot.data_ptr<int>(), dst_slot.data_ptr<int>(), rot.data_ptr<uint8_t>(),
      cos_n.data_ptr<float>(), sin_n.data_ptr<float>());
  FAK_CUDA_CHECK(cudaGetLastError());
}
