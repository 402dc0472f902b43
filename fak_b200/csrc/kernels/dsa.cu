// DeepSeek-style sparse attention (GLM-MoE-DSA): a learned indexer scores every cached key, the
// top-k keys are selected, and attention runs over the selected keys only (MLA: key width kd and
// value width vd differ).
//
// k_dsa_index_score  score[k] = sum_h w[h] * relu(scale * <iq[h], ik[k]>), keys k > qpos masked to
//                    -inf.  One warp per key; each lane owns heads h = lane, lane + 32, ...; the
//                    per-head dot and the head sum accumulate in double so the discrete selection
//                    is stable against reduction order.
// k_dsa_topk         one CTA: (score, position) pairs of the valid keys are bitonic-sorted in
//                    shared memory (score descending, lower position first on ties) and the first
//                    topk positions written out.  Up to kDsaMaxKeys keys.
// k_dsa_sparse_attend one CTA per query head, 4 warps: each warp streams a quarter of the selected
//                    keys straight from the cache rows (no host gather), keeps an online softmax
//                    (running max, sum, vd-wide accumulator in registers), and the warps merge in
//                    shared memory.
// Reference: k_dsa_index_score / k_dsa_index_topk / k_dsa_sparse_attend
// (internal/compute/cuda_kernels.cu:773-907), which score, select and attend the same way with a
// host-side gather and one block per key / repeated max passes.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "common.cuh"

namespace {

constexpr int kDsaMaxKeys = 16384;   // bitonic sort capacity: 16384 x 12 bytes of shared memory
constexpr int kAttnMaxV = 512;       // value width held in registers (16 per lane)

__global__ void k_dsa_index_score(const float* __restrict__ iq, const float* __restrict__ ik,
                                  const float* __restrict__ w, double* __restrict__ score, int n_keys, int nh,
                                  int dim, int qpos, double scale) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= n_keys) return;
  const int k = warp;
  double acc = 0.0;
  if (k <= qpos) {
    const float* key = ik + (int64_t)k * dim;
    for (int h = lane; h < nh; h += 32) {
      const float* q = iq + (int64_t)h * dim;
      double d = 0.0;
      for (int i = 0; i < dim; i++) d += (double)q[i] * (double)key[i];
      const double s = d * scale;
      acc += (double)w[h] * (s > 0.0 ? s : 0.0);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) score[k] = k <= qpos ? acc : -INFINITY;
}

// total order: higher score first, then lower position
FAK_DEV bool dsa_before(double a, int ia, double b, int ib) { return a > b || (a == b && ia < ib); }

__global__ void k_dsa_topk(const double* __restrict__ score, int n_valid, int n_pow2, int topk,
                           int* __restrict__ sel, int* __restrict__ count) {
  extern __shared__ __align__(16) uint8_t smem[];
  double* v = reinterpret_cast<double*>(smem);
  int* idx = reinterpret_cast<int*>(v + n_pow2);
  for (int i = threadIdx.x; i < n_pow2; i += blockDim.x) {
    v[i] = i < n_valid ? score[i] : -INFINITY;
    idx[i] = i < n_valid ? i : 0x7fffffff;
  }
  __syncthreads();
  for (int size = 2; size <= n_pow2; size <<= 1) {
    for (int stride = size >> 1; stride > 0; stride >>= 1) {
      for (int t = threadIdx.x; t < n_pow2 / 2; t += blockDim.x) {
        const int lo = 2 * stride * (t / stride) + (t % stride), hi = lo + stride;
        const bool up = (lo & size) == 0;   // this run sorts "before-first" when up
        const bool swap = up ? dsa_before(v[hi], idx[hi], v[lo], idx[lo]) : dsa_before(v[lo], idx[lo], v[hi], idx[hi]);
        if (swap) {
          const double tv = v[lo]; v[lo] = v[hi]; v[hi] = tv;
          const int ti = idx[lo]; idx[lo] = idx[hi]; idx[hi] = ti;
        }
      }
      __syncthreads();
    }
  }
  const int n = min(topk, n_valid);
  for (int i = threadIdx.x; i < n; i += blockDim.x) sel[i] = idx[i];
  if (threadIdx.x == 0) *count = n;
}

// q [H, kd]; kc [n_keys, H, kd]; vc [n_keys, H, vd]; sel [n_sel]; out [H, vd]
__global__ void __launch_bounds__(128) k_dsa_sparse_attend(const float* __restrict__ q, const float* __restrict__ kc,
                                                           const float* __restrict__ vc, const int* __restrict__ sel,
                                                           const int* __restrict__ n_sel_p, int n_keys, int H, int kd,
                                                           int vd, float scale, float* __restrict__ out) {
  constexpr int NV = kAttnMaxV / 32;
  __shared__ float s_m[4], s_l[4];
  __shared__ float s_acc[4][kAttnMaxV];
  const int h = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_sel = *n_sel_p;
  const float* qh = q + (int64_t)h * kd;
  float m = -INFINITY, l = 0.f, acc[NV];
#pragma unroll
  for (int i = 0; i < NV; i++) acc[i] = 0.f;
  for (int s = warp; s < n_sel; s += 4) {
    const int key = sel[s];
    if ((unsigned)key >= (unsigned)n_keys) continue;   // not a cached position: skipped
    const float* kr = kc + ((int64_t)key * H + h) * kd;
    float d = 0.f;
    for (int i = lane; i < kd; i += 32) d += qh[i] * kr[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    const float sc = d * scale;
    const float mn = fmaxf(m, sc);
    const float corr = __expf(m - mn), p = __expf(sc - mn);
    l = l * corr + p;
    const float* vr = vc + ((int64_t)key * H + h) * vd;
#pragma unroll
    for (int i = 0; i < NV; i++) {
      const int c = lane + 32 * i;
      acc[i] = acc[i] * corr + (c < vd ? p * vr[c] : 0.f);
    }
    m = mn;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
#pragma unroll
  for (int i = 0; i < NV; i++) s_acc[warp][lane + 32 * i] = acc[i];
  __syncthreads();
  float mx = fmaxf(fmaxf(s_m[0], s_m[1]), fmaxf(s_m[2], s_m[3]));
  float f[4], lt = 0.f;
#pragma unroll
  for (int w = 0; w < 4; w++) {
    f[w] = s_m[w] == -INFINITY ? 0.f : __expf(s_m[w] - mx);
    lt += s_l[w] * f[w];
  }
  const float inv = lt > 0.f ? 1.f / lt : 0.f;
  for (int c = threadIdx.x; c < vd; c += 128)
    out[(int64_t)h * vd + c] = (s_acc[0][c] * f[0] + s_acc[1][c] * f[1] + s_acc[2][c] * f[2] + s_acc[3][c] * f[3]) * inv;
}

}  // namespace

// Index scores [n_keys] f64 of one query: iq [nh, dim], ik [n_keys, dim], w [nh] (f32).
torch::Tensor dsa_index_score(torch::Tensor iq, torch::Tensor ik, torch::Tensor w, int64_t qpos, double scale) {
  TORCH_CHECK(iq.is_cuda() && iq.scalar_type() == torch::kFloat32 && iq.dim() == 2 && iq.is_contiguous(), "iq [nh, dim]");
  TORCH_CHECK(ik.scalar_type() == torch::kFloat32 && ik.dim() == 2 && ik.size(1) == iq.size(1) && ik.is_contiguous(),
              "ik [n_keys, dim]");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.numel() == iq.size(0), "w [nh]");
  const int n_keys = (int)ik.size(0);
  auto score = torch::empty({n_keys}, iq.options().dtype(torch::kFloat64));
  if (n_keys == 0) return score;
  const int threads = 256;
  k_dsa_index_score<<<(n_keys * 32 + threads - 1) / threads, threads, 0, at::cuda::getCurrentCUDAStream()>>>(
      iq.data_ptr<float>(), ik.data_ptr<float>(), w.data_ptr<float>(), score.data_ptr<double>(), n_keys,
      (int)iq.size(0), (int)iq.size(1), (int)qpos, scale);
  FAK_CUDA_CHECK(cudaGetLastError());
  return score;
}

// Top-k positions of the keys 0..qpos (score descending, lower position first): (sel [topk] int32,
// count [1] int32) -- count = min(topk, qpos + 1).
std::vector<torch::Tensor> dsa_topk(torch::Tensor score, int64_t qpos, int64_t topk) {
  TORCH_CHECK(score.is_cuda() && score.scalar_type() == torch::kFloat64 && score.dim() == 1, "score [n] f64");
  const int n_valid = (int)std::min<int64_t>(qpos + 1, score.numel());
  TORCH_CHECK(n_valid <= kDsaMaxKeys, "dsa_topk: more than ", kDsaMaxKeys, " candidate keys");
  TORCH_CHECK(topk >= 1, "dsa_topk: topk >= 1");
  auto opts = score.options().dtype(torch::kInt32);
  auto sel = torch::full({topk}, -1, opts);
  auto count = torch::zeros({1}, opts);
  if (n_valid <= 0) return {sel, count};
  int n_pow2 = 1;
  while (n_pow2 < n_valid) n_pow2 <<= 1;
  const size_t smem = (size_t)n_pow2 * (sizeof(double) + sizeof(int));
  FAK_CUDA_CHECK(cudaFuncSetAttribute(k_dsa_topk, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  k_dsa_topk<<<1, 1024, smem, at::cuda::getCurrentCUDAStream()>>>(score.data_ptr<double>(), n_valid, n_pow2,
                                                                   (int)topk, sel.data_ptr<int>(), count.data_ptr<int>());
  FAK_CUDA_CHECK(cudaGetLastError());
  return {sel, count};
}

// Attention of one query over selected keys: q [H, kd], k_cache [n_keys, H, kd], v_cache
// [n_keys, H, vd], sel [>= count] int32 positions, count [1] int32 (device) -> out [H, vd] f32.
torch::Tensor dsa_sparse_attend(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor sel,
                                torch::Tensor count, double scale) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kFloat32 && q.dim() == 2 && q.is_contiguous(), "q [H, kd]");
  const int H = (int)q.size(0), kd = (int)q.size(1);
  TORCH_CHECK(k_cache.scalar_type() == torch::kFloat32 && k_cache.dim() == 3 && k_cache.size(1) == H &&
                  k_cache.size(2) == kd && k_cache.is_contiguous(), "k_cache [n, H, kd]");
  TORCH_CHECK(v_cache.scalar_type() == torch::kFloat32 && v_cache.dim() == 3 && v_cache.size(1) == H &&
                  v_cache.size(0) == k_cache.size(0) && v_cache.is_contiguous(), "v_cache [n, H, vd]");
  const int vd = (int)v_cache.size(2);
  TORCH_CHECK(vd <= kAttnMaxV, "dsa_sparse_attend: value width <= ", kAttnMaxV);
  TORCH_CHECK(sel.scalar_type() == torch::kInt32 && count.scalar_type() == torch::kInt32 && count.numel() == 1,
              "sel / count int32");
  auto out = torch::empty({H, vd}, q.options());
  k_dsa_sparse_attend<<<H, 128, 0, at::cuda::getCurrentCUDAStream()>>>(
      q.data_ptr<float>(), k_cache.data_ptr<float>(), v_cache.data_ptr<float>(), sel.data_ptr<int>(),
      count.data_ptr<int>(), (int)k_cache.size(0), H, kd, vd, (float)scale, out.data_ptr<float>());
  FAK_CUDA_CHECK(cudaGetLastError());
  return out;
}
