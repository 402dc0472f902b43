// Token sampler on the device: logit bias, frequency / presence penalties, temperature, top-k, top-p,
// and a counter-based random draw, one CTA per row -- so a decode step with sampled lanes stays one
// CUDA graph with one token readback per step.
//
// Semantics (reference: internal/agent/inkernel_sampling.go:21-185):
//   eff[i]  = logit[i] + clamp(bias[i], -100, 100) - (freq * count[i] + pres * (count[i] > 0))
//   T <= 0  -> the first index of max(eff)            (greedy)
//   else    x = eff / T; top-k keeps the k largest x (ties at the k-th value kept); top-p keeps the
//           smallest set of largest-probability tokens whose mass reaches top_p of the (top-k)
//           total, the most likely token always kept (ties at the boundary value kept); a uniform
//           draw r in [0, kept mass) picks the token whose cumulative kept mass, walked in index
//           order, first exceeds r.
// Probabilities are integer weights w[i] = floor(exp(x[i] - max x) * 2^32) (so a token 2^-32 less
// likely than the best one is never drawn), summed in uint64 with integer atomics: the selection
// and the draw are exact integer arithmetic, identical on every run and on every tensor-parallel
// rank that samples the same gathered row.
//
// Selection by value uses radix search over the order-preserving 32-bit key of x: top-k finds the
// key of the k-th largest element (per-digit counts, most significant digit first), top-p the key
// where the running mass from the top first reaches the target (per-digit mass histograms); four
// passes of 8 bits each, shared-memory histograms, no sort.
//
// Random numbers: Philox-4x32 with 10 rounds (Salmon, Moraes, Dror and Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC 2011), key = the request's 64-bit seed, counter = (tokens it has
// generated so far, 0, 0, 0): the draw depends on the request alone, never on its batch.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "common.cuh"

using namespace fak;

namespace {

constexpr int kThreads = 1024;
constexpr float kBiasClamp = 100.f;
using u64 = unsigned long long;

// Per-row parameters, 10 int32 words (as the host packs them).
struct SampParam {
  float temperature;  // <= 0: greedy
  int top_k;          // <= 0 or >= V: off
  float top_p;        // >= 1 or <= 0: off
  float freq_pen;
  float pres_pen;
  int bias_off;       // this row's entries [bias_off, bias_off + bias_n) of the bias lists
  int bias_n;
  uint32_t seed_lo, seed_hi;
  uint32_t step;      // tokens generated so far (the draw's counter); the kernel advances it
};
static_assert(sizeof(SampParam) == 40, "SampParam is 10 words");

FAK_DEV uint32_t mulhilo(uint32_t a, uint32_t b, uint32_t& hi) {
  const u64 p = (u64)a * b;
  hi = (uint32_t)(p >> 32);
  return (uint32_t)p;
}

// Philox-4x32-10 (SC 2011): multipliers 0xD2511F53 / 0xCD9E8D57, Weyl key increments
// 0x9E3779B9 / 0xBB67AE85.
FAK_DEV uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; r++) {
    uint32_t hi0, hi1;
    const uint32_t lo0 = mulhilo(0xD2511F53u, c.x, hi0);
    const uint32_t lo1 = mulhilo(0xCD9E8D57u, c.z, hi1);
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
    k.x += 0x9E3779B9u;
    k.y += 0xBB67AE85u;
  }
  return c;
}

// order-preserving key of a float (larger float -> larger key)
FAK_DEV uint32_t fkey(float f) {
  const uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

FAK_DEV uint32_t weight(float x, float m) {
  // exp(x - m) in (0, 1] as a 32-bit fixed-point fraction; x = -inf (masked) -> 0
  const float e = __expf(x - m);
  const float s = e * 4294967296.0f;
  return s >= 4294967295.0f ? 0xffffffffu : (uint32_t)s;
}

template <typename T>
FAK_DEV T block_reduce_sum(T v, T* red) {
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();
  if (lane == 0) red[w] = v;
  __syncthreads();
  T s = 0;
  if (threadIdx.x < 32) {
    s = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : (T)0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (threadIdx.x == 0) red[0] = s;
  }
  __syncthreads();
  s = red[0];
  __syncthreads();
  return s;
}

__global__ void __launch_bounds__(kThreads, 1)
k_sample_rows(float* __restrict__ logits, int64_t ld, int V, SampParam* __restrict__ params,
              const int* __restrict__ bias_tok, const float* __restrict__ bias_val, int* __restrict__ counts,
              int64_t ldc, int* __restrict__ out, float softcap) {
  pdl_wait();
  const int b = blockIdx.x;
  float* x = logits + (int64_t)b * ld;
  int* cnt = counts ? counts + (int64_t)b * ldc : nullptr;
  const SampParam P = params[b];
  __shared__ u64 hist[256];
  __shared__ u64 red64[32];
  __shared__ float redf[32];
  __shared__ int redi[32];
  __shared__ uint32_t s_key, s_digit_rest;
  __shared__ u64 s_above;
  const int tid = threadIdx.x;

  // 1. final-logit soft-cap (Gemma-2: cap * tanh(logit / cap)), then penalties (from this row's
  //    generated-token counts) and the clamped logit bias, in place
  if (softcap > 0.f) {
    for (int i = tid; i < V; i += kThreads) x[i] = softcap * tanhf(x[i] / softcap);
    __syncthreads();
  }
  if (cnt != nullptr && (P.freq_pen != 0.f || P.pres_pen != 0.f)) {
    for (int i = tid; i < V; i += kThreads) {
      const int c = cnt[i];
      if (c > 0) x[i] -= P.freq_pen * (float)c + P.pres_pen;
    }
  }
  __syncthreads();
  for (int j = tid; j < P.bias_n; j += kThreads) {
    const int t = bias_tok[P.bias_off + j];
    if (t >= 0 && t < V) x[t] += fminf(kBiasClamp, fmaxf(-kBiasClamp, bias_val[P.bias_off + j]));
  }
  __syncthreads();

  // 2. max (and its first index, the greedy answer)
  float best = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = tid; i < V; i += kThreads) {
    const float v = x[i];
    if (v > best) { best = v; bi = i; }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
  }
  if ((tid & 31) == 0) { redf[tid >> 5] = best; redi[tid >> 5] = bi; }
  __syncthreads();
  if (tid == 0) {
    for (int w = 1; w < kThreads / 32; w++)
      if (redf[w] > redf[0] || (redf[w] == redf[0] && redi[w] < redi[0])) { redf[0] = redf[w]; redi[0] = redi[w]; }
  }
  __syncthreads();
  const float vmax = redf[0];
  const int argmax = redi[0] == 0x7fffffff ? 0 : redi[0];
  int token = argmax;

  if (P.temperature > 0.f && vmax > -INFINITY) {
    const float invT = 1.f / P.temperature;
    const float m = vmax * invT;
    // 3. top-k: key of the k-th largest x (ties at that value kept)
    uint32_t kth = 0;   // keep keys >= kth
    if (P.top_k > 0 && P.top_k < V) {
      uint32_t prefix = 0, need = (uint32_t)P.top_k;
      for (int pass = 0; pass < 4; pass++) {
        const int shift = 24 - 8 * pass;
        const uint32_t hmask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
        for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < V; i += kThreads) {
          const uint32_t k = fkey(x[i] * invT);
          if ((k & hmask) == prefix) atomicAdd(&hist[(k >> shift) & 255], 1ull);
        }
        __syncthreads();
        if (tid == 0) {
          u64 cum = 0;
          int d = 255;
          for (; d > 0; d--) {
            if (cum + hist[d] >= need) break;
            cum += hist[d];
          }
          s_key = prefix | ((uint32_t)d << shift);
          s_digit_rest = need - (uint32_t)cum;
        }
        __syncthreads();
        prefix = s_key;
        need = s_digit_rest;
        __syncthreads();
      }
      kth = prefix;
    }
    // kept mass after top-k
    u64 part = 0;
    for (int i = tid; i < V; i += kThreads) {
      const float xv = x[i] * invT;
      if (fkey(xv) >= kth) part += weight(xv, m);
    }
    const u64 total_k = block_reduce_sum<u64>(part, red64);
    // 4. top-p: the key where the running mass from the top first reaches top_p * total_k
    uint32_t pth = 0;
    if (P.top_p > 0.f && P.top_p < 1.f) {
      const u64 target = (u64)((double)P.top_p * (double)total_k);
      uint32_t prefix = 0;
      u64 above = 0;   // mass of keys above the current prefix range
      for (int pass = 0; pass < 4; pass++) {
        const int shift = 24 - 8 * pass;
        const uint32_t hmask = pass == 0 ? 0u : (0xffffffffu << (shift + 8));
        for (int i = tid; i < 256; i += kThreads) hist[i] = 0;
        __syncthreads();
        for (int i = tid; i < V; i += kThreads) {
          const float xv = x[i] * invT;
          const uint32_t k = fkey(xv);
          if (k >= kth && (k & hmask) == prefix)
            atomicAdd(&hist[(k >> shift) & 255],
                      (u64)weight(xv, m));
        }
        __syncthreads();
        if (tid == 0) {
          u64 cum = above;
          int d = 255;
          for (; d > 0; d--) {
            if (hist[d] != 0 && cum + hist[d] >= target) break;
            cum += hist[d];
          }
          s_key = prefix | ((uint32_t)d << shift);
          s_above = cum;
        }
        __syncthreads();
        prefix = s_key;
        above = s_above;
        __syncthreads();
      }
      pth = prefix;
    }
    const uint32_t thr = kth > pth ? kth : pth;
    // 5. the draw: per-thread contiguous chunks walked in index order
    const int chunk = (V + kThreads - 1) / kThreads;
    const int i0 = tid * chunk, i1 = min(V, i0 + chunk);
    u64 mine = 0;
    for (int i = i0; i < i1; i++) {
      const float xv = x[i] * invT;
      if (fkey(xv) >= thr) mine += weight(xv, m);
    }
    // exclusive prefix over threads (warp scan, then over warps)
    u64 incl = mine;
    const int lane = tid & 31, w = tid >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const u64 y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    if (lane == 31) red64[w] = incl;
    __syncthreads();
    if (tid == 0) {
      u64 run = 0;
      for (int j = 0; j < kThreads / 32; j++) {
        const u64 t = red64[j];
        red64[j] = run;
        run += t;
      }
      s_above = run;   // total kept mass
    }
    __syncthreads();
    const u64 excl = red64[w] + incl - mine;
    const u64 S = s_above;
    const uint4 rnd = philox4x32_10(make_uint4(P.step, 0u, 0u, 0u), make_uint2(P.seed_lo, P.seed_hi));
    const u64 u = ((u64)rnd.x << 32) | rnd.y;
    const u64 r = S ? __umul64hi(u, S) : 0;   // uniform in [0, S)
    if (tid == 0) redi[0] = -1;
    __syncthreads();
    if (S > 0 && mine > 0 && r >= excl && r < excl + mine) {
      u64 acc = excl;
      int pick = -1;
      for (int i = i0; i < i1; i++) {
        const float xv = x[i] * invT;
        if (fkey(xv) < thr) continue;
        acc += weight(xv, m);
        pick = i;
        if (acc > r) break;
      }
      redi[0] = pick;
    }
    __syncthreads();
    token = redi[0] >= 0 ? redi[0] : argmax;
  }
  if (tid == 0) {
    out[b] = token;
    if (cnt != nullptr) cnt[token] += 1;
    params[b].step = P.step + 1;
  }
  pdl_launch_dependents();
}

}  // namespace

// logits [B, >=V] f32 (modified in place: penalties and bias); params int32 [B, 10] (SampParam words,
// step advanced); bias_tok / bias_val flat lists (params index them); counts int32 [B, >=V] or none
// (penalties need it; incremented at the drawn token); out int32 [B].
void sample_rows(torch::Tensor logits, int64_t V, torch::Tensor params, torch::Tensor bias_tok, torch::Tensor bias_val,
                 c10::optional<torch::Tensor> counts, torch::Tensor out, int64_t B, double softcap) {
  TORCH_CHECK(logits.is_cuda() && logits.scalar_type() == torch::kFloat32 && logits.dim() == 2 &&
                  logits.stride(1) == 1 && logits.size(0) >= B && logits.size(1) >= V, "sample_rows: logits");
  TORCH_CHECK(params.scalar_type() == torch::kInt32 && params.is_contiguous() && params.numel() >= B * 10,
              "sample_rows: params int32 [B, 10]");
  TORCH_CHECK(bias_tok.scalar_type() == torch::kInt32 && bias_val.scalar_type() == torch::kFloat32 &&
                  bias_tok.numel() == bias_val.numel(), "sample_rows: bias lists");
  TORCH_CHECK(out.scalar_type() == torch::kInt32 && out.numel() >= B, "sample_rows: out");
  int* cp = nullptr;
  int64_t ldc = 0;
  if (counts.has_value()) {
    TORCH_CHECK(counts->scalar_type() == torch::kInt32 && counts->dim() == 2 && counts->stride(1) == 1 &&
                    counts->size(0) >= B && counts->size(1) >= V, "sample_rows: counts [B, >=V] int32");
    cp = counts->data_ptr<int>();
    ldc = counts->stride(0);
  }
  if (B <= 0) return;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)B);
  cfg.blockDim = dim3(kThreads);
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_sample_rows, logits.data_ptr<float>(), (int64_t)logits.stride(0), (int)V,
                                    reinterpret_cast<SampParam*>(params.data_ptr<int>()),
                                    (const int*)bias_tok.data_ptr<int>(), (const float*)bias_val.data_ptr<float>(), cp,
                                    ldc, out.data_ptr<int>(), (float)softcap));
}

// Philox-4x32-10 of one (counter, key) pair on the host, the same arithmetic as the device rounds
// (for known-answer tests of the generator).
torch::Tensor philox4x32_10_host(std::vector<int64_t> ctr, std::vector<int64_t> key) {
  TORCH_CHECK(ctr.size() == 4 && key.size() == 2, "philox: 4 counter words, 2 key words");
  uint32_t c[4], k[2];
  for (int i = 0; i < 4; i++) c[i] = (uint32_t)ctr[i];
  for (int i = 0; i < 2; i++) k[i] = (uint32_t)key[i];
  for (int r = 0; r < 10; r++) {
    const u64 p0 = (u64)0xD2511F53u * c[0], p1 = (u64)0xCD9E8D57u * c[2];
    const uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k[0], n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k[1];
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
    k[0] += 0x9E3779B9u;
    k[1] += 0xBB67AE85u;
  }
  auto t = torch::empty({4}, torch::kInt64);
  for (int i = 0; i < 4; i++) t.data_ptr<int64_t>()[i] = c[i];
  return t;
}
