// Small fused kernels around the GEMMs: embedding gather (dequantizing the GGML rows of the
// token table), RoPE + optional per-head q/k RMSNorm + paged KV append, RMSNorm to bf16, and
// greedy argmax.
//
// RoPE uses a precomputed cos/sin table whose angles were evaluated in float64, matching the
// reference's double-precision angle (internal/compute/cuda_kernels.cu:551-567); the KV append
// writes through a slot mapping (page*16 + offset) instead of a contiguous offset
// (reference k_copyrow, cuda_kernels.cu:599-605), which is what lets pages be shared.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "common.cuh"

using namespace fak;

namespace {

constexpr int PAGE = 16;

FAK_DEV float dequant_one(const uint8_t* row, int qtype, int c) {
  if (qtype == QT_Q8_0) {
    const uint8_t* blk = row + (c >> 5) * 34;
    return half_bits_to_float(ld_u16(blk)) * (float)(int8_t)blk[2 + (c & 31)];
  }
  if (qtype == QT_Q4_K) {
    const uint8_t* blk = row + (c >> 8) * 144;
    int e = c & 255, j = e >> 5, l = e & 31;
    const uint8_t* s = blk + 4;
    int sc, m;
    if (j < 4) { sc = s[j] & 63; m = s[j + 4] & 63; }
    else { sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4); m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4); }
    int q = (blk[16 + (j >> 1) * 32 + l] >> ((j & 1) * 4)) & 15;
    return half_bits_to_float(ld_u16(blk)) * (float)sc * (float)q - half_bits_to_float(ld_u16(blk + 2)) * (float)m;
  }
  if (qtype == QT_Q6_K) {
    const uint8_t* blk = row + (c >> 8) * 210;
    int e = c & 255, n = e >> 7, k = (e & 127) >> 5, l = e & 31;
    int q = ((blk[n * 64 + (k & 1) * 32 + l] >> ((k >> 1) * 4)) & 15) | (((blk[128 + n * 32 + l] >> (2 * k)) & 3) << 4);
    return half_bits_to_float(ld_u16(blk + 208)) * (float)(int8_t)blk[192 + (e >> 4)] * (float)(q - 32);
  }
  if (qtype == QT_F32) return reinterpret_cast<const float*>(row)[c];
  if (qtype == QT_F16) return __half2float(reinterpret_cast<const __half*>(row)[c]);
  if (qtype == QT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(row)[c]);
  return 0.f;
}

__global__ void k_embed(const uint8_t* __restrict__ table, int qtype, int64_t pitch, int V, int d,
                        const int* __restrict__ ids, float* __restrict__ out_f32, __nv_bfloat16* __restrict__ out_bf16,
                        int* __restrict__ err, float scale) {
  pdl_wait();
  int t = blockIdx.x;
  int id = ids[t];
  if (id < 0 || id >= V) {
    if (threadIdx.x == 0 && blockIdx.y == 0) report_error(err, 2);
    id = 0;
  }
  const uint8_t* row = table + (int64_t)id * pitch;
  // grid.y spreads a row over CTAs: one element per thread, so every element's block reads of a
  // row are in flight at once (decode gathers only a few rows)
  for (int c = blockIdx.y * blockDim.x + threadIdx.x; c < d; c += blockDim.x * gridDim.y) {
    float v = dequant_one(row, qtype, c) * scale;   // scale: embedding multiplier (Gemma: sqrt(d))
    if (out_f32) out_f32[(int64_t)t * d + c] = v;
    if (out_bf16) out_bf16[(int64_t)t * d + c] = __float2bfloat16_rn(v);
  }
  pdl_launch_dependents();
}

// One warp per head. qkv [T, (H + 2*Hkv) * D] f32 (row stride ld).  Lane holds dims
// {lane + 32*i}; rotate_half pairs (j, j + D/2) land in the same lane.
template <int D>
__global__ void k_rope_kv(const float* __restrict__ qkv, int64_t ld, const int* __restrict__ pos,
                          const int* __restrict__ slot, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                          int H, int Hkv, const float* __restrict__ qn, const float* __restrict__ kn, float eps,
                          float* __restrict__ q_f32, __nv_bfloat16* __restrict__ q_bf16,
                          __nv_bfloat16* __restrict__ kc, __nv_bfloat16* __restrict__ vc, int n_pages, int n_pos) {
  constexpr int PER = D / 32;  // values per lane
  constexpr int HALF = D / 2;
  pdl_wait();
  const int t = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  // positions past the RoPE table are clamped (the engine never issues them; the clamp keeps a
  // bad position from reading outside the table)
  const int p = min(max(pos[t], 0), n_pos - 1);
  const int sl = slot[t];
  const int page = sl / PAGE, off = sl % PAGE;
  const float* row = qkv + (int64_t)t * ld;
  // grid.y spreads the heads of a token over several CTAs (decode has only a few tokens)
  for (int hh = blockIdx.y * nw + warp; hh < H + 2 * Hkv; hh += nw * gridDim.y) {
    const bool is_q = hh < H, is_k = !is_q && hh < H + Hkv;
    const float* src = row + (int64_t)hh * D;
    float v[PER];
#pragma unroll
    for (int i = 0; i < PER; i++) v[i] = src[lane + 32 * i];
    if (is_q || is_k) {
      const float* g = is_q ? qn : kn;
      if (g) {
        float ss = 0.f;
#pragma unroll
        for (int i = 0; i < PER; i++) ss += v[i] * v[i];
        ss = warp_sum(ss);
        float inv = rsqrtf(ss / (float)D + eps);
#pragma unroll
        for (int i = 0; i < PER; i++) v[i] = v[i] * inv * g[lane + 32 * i];
      }
      float r[PER];
#pragma unroll
      for (int i = 0; i < PER; i++) {
        int dim = lane + 32 * i;
        int j = dim % HALF;
        float c = cos_t[(int64_t)p * HALF + j], s = sin_t[(int64_t)p * HALF + j];
        // partner value lives in the same lane, PER/2 slots away
        float other = v[(i + PER / 2) % PER];
        r[i] = dim < HALF ? v[i] * c - other * s : v[i] * c + other * s;
      }
#pragma unroll
      for (int i = 0; i < PER; i++) v[i] = r[i];
    }
    if (is_q) {
#pragma unroll
      for (int i = 0; i < PER; i++) {
        int64_t oi = ((int64_t)t * H + hh) * D + lane + 32 * i;
        if (q_f32) q_f32[oi] = v[i];
        if (q_bf16) q_bf16[oi] = __float2bfloat16_rn(v[i]);
      }
    } else if (sl >= 0 && page < n_pages) {
      int kvh = is_k ? hh - H : hh - H - Hkv;
      __nv_bfloat16* dst = (is_k ? kc : vc) + (((int64_t)page * Hkv + kvh) * PAGE + off) * D;
#pragma unroll
      for (int i = 0; i < PER; i++) dst[lane + 32 * i] = __float2bfloat16_rn(v[i]);
    }
  }
  pdl_launch_dependents();
}

// RMSNorm rows of an fp32 matrix into bf16 (the prefill GEMM operand).
__global__ void k_rmsnorm_bf16(const float* __restrict__ x, int64_t ldx, const float* __restrict__ w, float eps, int d,
                               __nv_bfloat16* __restrict__ y, int64_t ldy) {
  pdl_wait();
  const int r = blockIdx.x;
  const float* xr = x + (int64_t)r * ldx;
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) ss += xr[i] * xr[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  float inv = rsqrtf(red[0] / (float)d + eps);
  pdl_launch_dependents();
  for (int i = threadIdx.x; i < d; i += blockDim.x) y[(int64_t)r * ldy + i] = __float2bfloat16_rn(xr[i] * inv * w[i]);
}

// first-index argmax per row (ties resolve to the lowest id, as the reference's k_argmax)
__global__ void k_argmax(const float* __restrict__ logits, int64_t ld, int V, int* __restrict__ out) {
  pdl_wait();
  const int r = blockIdx.x;
  const float* x = logits + (int64_t)r * ld;
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = threadIdx.x; i < V; i += blockDim.x) {
    float v = x[i];
    if (v > best || (v == best && i < bi)) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float ov = __shfl_xor_sync(0xffffffffu, best, o);
    int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  __shared__ float sv[32];
  __shared__ int si[32];
  if ((threadIdx.x & 31) == 0) { sv[threadIdx.x >> 5] = best; si[threadIdx.x >> 5] = bi; }
  __syncthreads();
  if (threadIdx.x < 32) {
    int nw = blockDim.x >> 5;
    best = threadIdx.x < nw ? sv[threadIdx.x] : -INFINITY;
    bi = threadIdx.x < nw ? si[threadIdx.x] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, best, o);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (threadIdx.x == 0) out[r] = bi == 0x7fffffff ? 0 : bi;
  }
  pdl_launch_dependents();
}

// Multi-CTA first-index argmax: grid (rows, chunks).  Each CTA folds its chunk into one packed
// 64-bit key per row (argmax_key: atomicMax keeps the largest value and, among equal values, the
// lowest index), and the last CTA of a row (ticket) writes the index and resets the key and ticket
// to zero.
constexpr int kArgmaxThreads = 256, kArgmaxPer = 4;   // a CTA's chunk: 256 x 4 x 4 = 4096 floats
template <bool VEC>
__global__ void k_argmax_chunks(const float* __restrict__ logits, int64_t ld, int V, int chunk,
                                unsigned long long* __restrict__ keys, int* __restrict__ tickets, int* __restrict__ out) {
  pdl_wait();
  const int r = blockIdx.x;
  const int i0 = blockIdx.y * chunk, i1 = min(V, i0 + chunk);
  const unsigned long long best = cta_best_key<VEC ? kArgmaxPer : 4 * kArgmaxPer, VEC>(logits + (int64_t)r * ld, i0, i1, 0u);
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    atomicMax(&keys[r], best);
    __threadfence();
    s_last = atomicAdd(&tickets[r], 1) == (int)gridDim.y - 1;
  }
  __syncthreads();
  pdl_launch_dependents();
  if (threadIdx.x == 0 && s_last) {
    __threadfence();
    const unsigned long long k = atomicExch(&keys[r], 0ull);
    out[r] = argmax_key_index(k);
    tickets[r] = 0;
  }
}

cudaLaunchAttribute g_attr[1];
cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, size_t smem = 0) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  g_attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  g_attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = g_attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

void embed(torch::Tensor table, int64_t qtype, int64_t pitch, int64_t V, int64_t d, torch::Tensor ids,
           c10::optional<torch::Tensor> out_f32, c10::optional<torch::Tensor> out_bf16,
           c10::optional<torch::Tensor> err, double scale) {
  TORCH_CHECK(table.is_cuda() && table.scalar_type() == torch::kUInt8, "table");
  TORCH_CHECK(ids.scalar_type() == torch::kInt32 && ids.is_contiguous(), "ids int32");
  int T = (int)ids.numel();
  if (T == 0) return;
  float* of = out_f32.has_value() ? out_f32->data_ptr<float>() : nullptr;
  __nv_bfloat16* ob = out_bf16.has_value() ? reinterpret_cast<__nv_bfloat16*>(out_bf16->data_ptr()) : nullptr;
  if (of) TORCH_CHECK(out_f32->is_contiguous() && out_f32->numel() >= (int64_t)T * d, "out_f32");
  if (ob) TORCH_CHECK(out_bf16->is_contiguous() && out_bf16->numel() >= (int64_t)T * d, "out_bf16");
  int* ep = err.has_value() ? err->data_ptr<int>() : nullptr;
  auto cfg = make_cfg(dim3(T, (unsigned)((d + 255) / 256)), dim3(256));
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_embed, (const uint8_t*)table.data_ptr<uint8_t>(), (int)qtype, pitch, (int)V,
                                    (int)d, (const int*)ids.data_ptr<int>(), of, ob, ep, (float)scale));
}

// x[t] += rmsnorm(y[t]) * w  (Gemma's sandwich norms: the attention / FFN output is normalised
// before the residual add).  One CTA of 256 threads per row; y and x rows of d floats.
__global__ void k_rmsnorm_add(const float* __restrict__ y, int64_t ldy, const float* __restrict__ w, float eps,
                              int d, float* __restrict__ x, int64_t ldx) {
  __shared__ float red[8];
  pdl_wait();
  const int t = blockIdx.x;
  const float* yr = y + (int64_t)t * ldy;
  float ss = 0.f;
  for (int c = threadIdx.x; c < d; c += blockDim.x) ss += yr[c] * yr[c];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < 8; i++) tot += red[i];
  const float inv = rsqrtf(tot / (float)d + eps);
  pdl_launch_dependents();
  float* xr = x + (int64_t)t * ldx;
  for (int c = threadIdx.x; c < d; c += blockDim.x) xr[c] += yr[c] * inv * w[c];
}

void rmsnorm_add(torch::Tensor y, torch::Tensor w, double eps, torch::Tensor x) {
  TORCH_CHECK(y.is_cuda() && y.scalar_type() == torch::kFloat32 && y.dim() == 2 && y.stride(1) == 1, "y [T, d] f32");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.dim() == 2 && x.stride(1) == 1 && x.size(0) >= y.size(0) &&
                  x.size(1) == y.size(1), "x [T, d] f32");
  TORCH_CHECK(w.scalar_type() == torch::kFloat32 && w.numel() == y.size(1), "w [d] f32");
  const int T = (int)y.size(0);
  if (T == 0) return;
  auto cfg = make_cfg(dim3(T), dim3(256));
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_rmsnorm_add, (const float*)y.data_ptr<float>(), (int64_t)y.stride(0),
                                    (const float*)w.data_ptr<float>(), (float)eps, (int)y.size(1), x.data_ptr<float>(),
                                    (int64_t)x.stride(0)));
}

void rope_kv(torch::Tensor qkv, torch::Tensor pos, torch::Tensor slot, torch::Tensor cos_t, torch::Tensor sin_t,
             int64_t H, int64_t Hkv, c10::optional<torch::Tensor> q_norm, c10::optional<torch::Tensor> k_norm, double eps,
             c10::optional<torch::Tensor> q_f32, c10::optional<torch::Tensor> q_bf16, torch::Tensor k_cache,
             torch::Tensor v_cache) {
  TORCH_CHECK(qkv.scalar_type() == torch::kFloat32 && qkv.dim() == 2 && qkv.stride(1) == 1, "qkv [T, *] f32");
  int T = (int)qkv.size(0);
  int D = (int)k_cache.size(3);
  TORCH_CHECK(k_cache.size(1) == Hkv && k_cache.size(2) == PAGE && k_cache.is_contiguous() && v_cache.is_contiguous(),
              "cache layout");
  TORCH_CHECK(qkv.size(1) >= (H + 2 * Hkv) * D, "qkv width");
  TORCH_CHECK(pos.scalar_type() == torch::kInt32 && slot.scalar_type() == torch::kInt32, "pos/slot int32");
  TORCH_CHECK(cos_t.scalar_type() == torch::kFloat32 && cos_t.size(1) == D / 2 && cos_t.size(0) >= 1 &&
                  sin_t.sizes() == cos_t.sizes(), "cos/sin table");
  if (T == 0) return;
  const float* qn = q_norm.has_value() ? q_norm->data_ptr<float>() : nullptr;
  const float* kn = k_norm.has_value() ? k_norm->data_ptr<float>() : nullptr;
  float* qf = q_f32.has_value() ? q_f32->data_ptr<float>() : nullptr;
  __nv_bfloat16* qb = q_bf16.has_value() ? reinterpret_cast<__nv_bfloat16*>(q_bf16->data_ptr()) : nullptr;
  const int heads = (int)(H + 2 * Hkv);
  auto cfg = make_cfg(dim3(T, T >= 64 ? 1 : (heads + 3) / 4), dim3(T >= 64 ? 256 : 128));
  int n_pages = (int)k_cache.size(0);
  auto launch = [&](auto kern) {
    FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, (const float*)qkv.data_ptr<float>(), (int64_t)qkv.stride(0),
                                      (const int*)pos.data_ptr<int>(), (const int*)slot.data_ptr<int>(),
                                      (const float*)cos_t.data_ptr<float>(), (const float*)sin_t.data_ptr<float>(),
                                      (int)H, (int)Hkv, qn, kn, (float)eps, qf, qb,
                                      (__nv_bfloat16*)k_cache.data_ptr(), (__nv_bfloat16*)v_cache.data_ptr(), n_pages,
                                      (int)cos_t.size(0)));
  };
  if (D == 128) launch(k_rope_kv<128>);
  else if (D == 64) launch(k_rope_kv<64>);
  else TORCH_CHECK(false, "head dim must be 64 or 128");
}

void rmsnorm_bf16(torch::Tensor x, torch::Tensor w, double eps, torch::Tensor y) {
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.dim() == 2 && x.stride(1) == 1, "x");
  TORCH_CHECK(y.scalar_type() == torch::kBFloat16 && y.dim() == 2 && y.stride(1) == 1, "y");
  int R = (int)x.size(0), d = (int)x.size(1);
  if (R == 0) return;
  auto cfg = make_cfg(dim3(R), dim3(256));
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_rmsnorm_bf16, (const float*)x.data_ptr<float>(), (int64_t)x.stride(0),
                                    (const float*)w.data_ptr<float>(), (float)eps, d,
                                    (__nv_bfloat16*)y.data_ptr(), (int64_t)y.stride(0)));
}

void argmax_rows(torch::Tensor logits, int64_t V, torch::Tensor out, c10::optional<torch::Tensor> keys,
                 c10::optional<torch::Tensor> tickets) {
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.dim() == 2 && logits.stride(1) == 1, "logits");
  TORCH_CHECK(out.scalar_type() == torch::kInt32, "out int32");
  int R = (int)logits.size(0);
  if (R == 0) return;
  if (keys.has_value()) {
    TORCH_CHECK(keys->scalar_type() == torch::kInt64 && keys->numel() >= R, "argmax: keys [R] int64");
    TORCH_CHECK(tickets.has_value() && tickets->scalar_type() == torch::kInt32 && tickets->numel() >= R,
                "argmax: tickets [R] int32");
    const int chunk = kArgmaxThreads * kArgmaxPer * 4;
    const bool vec = logits.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0;
    auto cfg = make_cfg(dim3(R, (unsigned)((V + chunk - 1) / chunk)), dim3(kArgmaxThreads));
    FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, vec ? k_argmax_chunks<true> : k_argmax_chunks<false>,
                                      (const float*)logits.data_ptr<float>(), (int64_t)logits.stride(0), (int)V, chunk,
                                      reinterpret_cast<unsigned long long*>(keys->data_ptr<int64_t>()),
                                      tickets->data_ptr<int>(), out.data_ptr<int>()));
    return;
  }
  auto cfg = make_cfg(dim3(R), dim3(1024));
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_argmax, (const float*)logits.data_ptr<float>(), (int64_t)logits.stride(0),
                                    (int)V, out.data_ptr<int>()));
}
