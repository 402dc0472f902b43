// Mixture-of-experts decode kernels: routing, per-expert token grouping, grouped quantized
// expert GEMV on the integer tensor cores, and the weighted combine.
//
// Router semantics match the reference (internal/model/moe.go:279-311): softmax over all
// experts, top-k, renormalised to sum 1 when norm_topk_prob.  Grouping is deterministic
// (tokens keep their order inside an expert's list), so the combine sums in a fixed order and
// batched == serial.
//
// The grouped GEMV processes work items (chunk, tile): a chunk is up to 8 (token, expert) pairs
// routed to the same expert, a tile 16 weight rows of that expert.  One CTA per work item: the
// tile's 16 rows move with one 1-D TMA bulk copy (experts are stored back to back, rows at the
// device pitch), the chunk's 8 activation rows are gathered with one bulk copy each, and the
// math is the same per-block-scaled int8 MMA as the dense decode GEMV.  The grid is sized for
// the worst case so the launch is graph-capturable; work items past the live chunk count exit.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "tc.cuh"

using namespace fak;

namespace {

constexpr int MAX_K = 16;  // top-k bound
constexpr int CH = 8;      // pairs per chunk (MMA N)

// ---------------------------------------------------------------------------------------------
// routing: one CTA per token.  x fp32 residual row -> RMSNorm(gamma) -> logits = W_r x (fp32) ->
// softmax -> top-k -> renorm.  Writes ids [T, k] and weights [T, k].
// ---------------------------------------------------------------------------------------------
// kind 0: softmax over every expert, then the top k (renormalised with norm_topk); kind 1 (gpt-oss):
// the top k logits, then a softmax over those k.  rbias (optional) is added to the logits first.
__global__ void k_moe_route(const float* __restrict__ x, int64_t ldx, const float* __restrict__ gamma, float eps,
                            const float* __restrict__ wr, int E, int d, int k, int norm_topk, int* __restrict__ ids,
                            float* __restrict__ wts, const float* __restrict__ rbias, int kind) {
  pdl_wait();
  extern __shared__ float rsm[];  // [d] normalized x | [E] logits
  float* xs = rsm;
  float* lg = rsm + d;
  const int t = blockIdx.x;
  const float* xr = x + (int64_t)t * ldx;
  __shared__ float red[32];
  float ss = 0.f;
  for (int i = threadIdx.x; i < d; i += blockDim.x) ss += xr[i] * xr[i];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (int)(blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)d + eps);
  for (int i = threadIdx.x; i < d; i += blockDim.x) xs[i] = xr[i] * inv * gamma[i];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int e = warp; e < E; e += nw) {
    const float* w = wr + (int64_t)e * d;
    float acc = 0.f;
    for (int i = lane; i < d; i += 32) acc += w[i] * xs[i];
    acc = warp_sum(acc);
    if (lane == 0) lg[e] = acc + (rbias ? rbias[e] : 0.f);
  }
  __syncthreads();
  if (threadIdx.x == 0 && kind == 1) {
    float sel_v[MAX_K];
    int sel_i[MAX_K];
    for (int j = 0; j < k; j++) {  // top-k logits in descending order, first index wins ties
      int bi = -1;
      float bv = -INFINITY;
      for (int e = 0; e < E; e++) {
        if (bi < 0 || lg[e] > bv) { bv = lg[e]; bi = e; }
      }
      sel_i[j] = bi;
      sel_v[j] = bv;
      lg[bi] = -INFINITY;   // chosen: never picked again
    }
    float s = 0.f;
    for (int j = 0; j < k; j++) s += __expf(sel_v[j] - sel_v[0]);
    for (int j = 0; j < k; j++) {
      ids[(int64_t)t * k + j] = sel_i[j];
      wts[(int64_t)t * k + j] = __expf(sel_v[j] - sel_v[0]) / s;
    }
  }
  if (threadIdx.x == 0 && kind == 0) {
    float mx = -INFINITY;
    for (int e = 0; e < E; e++) mx = fmaxf(mx, lg[e]);
    float s = 0.f;
    for (int e = 0; e < E; e++) {
      lg[e] = __expf(lg[e] - mx);
      s += lg[e];
    }
    float sel_w[MAX_K];
    int sel_i[MAX_K];
    float tot = 0.f;
    for (int j = 0; j < k; j++) {  // top-k, first index wins ties
      int bi = -1;
      float bv = -1.f;
      for (int e = 0; e < E; e++) {
        if (lg[e] > bv) { bv = lg[e]; bi = e; }
      }
      sel_i[j] = bi;
      sel_w[j] = bv / s;
      tot += sel_w[j];
      lg[bi] = -2.f;
    }
    for (int j = 0; j < k; j++) {
      ids[(int64_t)t * k + j] = sel_i[j];
      wts[(int64_t)t * k + j] = norm_topk ? sel_w[j] / tot : sel_w[j];
    }
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------------------------
// grouping: one CTA.  Pairs p = t*k + j.  Only experts in [e0, e0+E_local) are kept (expert
// parallelism).  Output chunks: chunk_expert[c] (local expert index), chunk_pairs[c][8] (pair ids,
// -1 = empty); n_chunks[0].  Deterministic: experts ascending, pairs ascending within an expert.
// ---------------------------------------------------------------------------------------------
__global__ void k_moe_group(const int* __restrict__ ids, int P, int e0, int E_local, int max_chunks,
                            int* __restrict__ chunk_expert, int* __restrict__ chunk_pairs, int* __restrict__ n_chunks) {
  pdl_wait();
  extern __shared__ int cnt_sm[];  // [E_local] counts, then [E_local] chunk offsets
  int* cnt = cnt_sm;
  int* off = cnt + E_local;
  for (int e = threadIdx.x; e < E_local; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < P; p += blockDim.x) {
    const int e = ids[p] - e0;
    if (e >= 0 && e < E_local) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int c = 0;
    for (int e = 0; e < E_local; e++) {
      off[e] = c;
      c += (cnt[e] + CH - 1) / CH;
    }
    n_chunks[0] = min(c, max_chunks);
  }
  __syncthreads();
  // each expert's pairs in ascending order: one thread per expert scans the pair list
  for (int e = threadIdx.x; e < E_local; e += blockDim.x) {
    int c = off[e], slot = 0;
    if (cnt[e] == 0) continue;
    for (int p = 0; p < P; p++) {
      if (ids[p] - e0 != e) continue;
      if (c < max_chunks) {
        if (slot == 0) {
          chunk_expert[c] = e;
          for (int s = 0; s < CH; s++) chunk_pairs[c * CH + s] = -1;
        }
        chunk_pairs[c * CH + slot] = p;
      }
      if (++slot == CH) { slot = 0; c++; }
    }
  }
  pdl_launch_dependents();
}

// ---------------------------------------------------------------------------------------------
// grouped GEMV (Q8_0 / Q4_K / Q6_K experts)
// ---------------------------------------------------------------------------------------------
FAK_DEV void mma_s8_16832(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
FAK_DEV uint32_t lds_u32_a2(const uint8_t* p) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if ((a & 3) == 0) return *reinterpret_cast<const uint32_t*>(p);
  const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
  return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
}
FAK_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          tc::smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(tc::smem_addr(bar))
      : "memory");
}

enum GEpi : int { GE_STORE = 0, GE_SWIGLU = 2 };

// Q8_0 experts (the MoE checkpoint format of the benchmark).  acts: int8 codes [rows, K] with
// (scale, sum) [rows, K/32]; act_row(pair) selects the activation row of a pair (the token for
// gate/up, the pair itself for down); output row = pair.
template <int ACT_BY_TOKEN>
__global__ void __launch_bounds__(256)
k_moe_qmmv_q8(const uint8_t* __restrict__ W, int rows_per_expert, int K, int64_t pitch,
              const int8_t* __restrict__ qx, const float2* __restrict__ ds, int topk,
              const int* __restrict__ chunk_expert, const int* __restrict__ chunk_pairs, const int* __restrict__ n_chunks,
              float* __restrict__ y, int64_t ldy, int epi, int* __restrict__ err) {
  extern __shared__ __align__(128) uint8_t gsm[];
  __shared__ uint64_t bar;
  __shared__ float red[8][32][4];
  const int tiles = rows_per_expert / 16;
  const int chunk = blockIdx.x / tiles, tile = blockIdx.x % tiles;
  pdl_wait();
  if (chunk >= n_chunks[0]) return;
  const int e = chunk_expert[chunk];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int64_t nblk = K >> 5;
  const int xs_stride = K + 32;
  uint8_t* wsm = gsm;                                   // [16][pitch]
  int8_t* xsm = reinterpret_cast<int8_t*>(gsm + 16 * pitch);  // [8][K + 32]
  float2* dsm = reinterpret_cast<float2*>(gsm + 16 * pitch + CH * xs_stride);  // [8][K/32]
  int pr[CH];
#pragma unroll
  for (int s = 0; s < CH; s++) pr[s] = chunk_pairs[chunk * CH + s];
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int nv = 0;
    for (int s = 0; s < CH; s++) nv += pr[s] >= 0;
    const uint32_t wbytes = (uint32_t)(16 * pitch);
    tc::mbar_arrive_expect_tx(&bar, wbytes + nv * (uint32_t)(K + K / 4));
    const uint8_t* wt = W + ((int64_t)e * rows_per_expert + (int64_t)tile * 16) * pitch;
    bulk_g2s(wsm, wt, wbytes, &bar);
    for (int s = 0; s < CH; s++) {
      if (pr[s] < 0) continue;
      const int64_t row = ACT_BY_TOKEN ? pr[s] / topk : pr[s];
      bulk_g2s(xsm + s * xs_stride, qx + row * K, (uint32_t)K, &bar);
      bulk_g2s(dsm + s * nblk, ds + row * nblk, (uint32_t)(K / 4), &bar);
    }
  }
  tc::mbar_wait(&bar, 0, err);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  const bool tok_ok = pr[g] >= 0;
  const int s0 = 2 * t, s1 = 2 * t + 1;
  const bool ok0 = pr[s0] >= 0, ok1 = pr[s1] >= 0;
  for (int64_t blk = warp; blk < nblk; blk += 8) {
    const uint8_t* pa = wsm + g * pitch + blk * 34;
    const uint8_t* pb = wsm + (g + 8) * pitch + blk * 34;
    const uint2 qa = make_uint2(lds_u32_a2(pa + 2 + 8 * t), lds_u32_a2(pa + 6 + 8 * t));
    const uint2 qb = make_uint2(lds_u32_a2(pb + 2 + 8 * t), lds_u32_a2(pb + 6 + 8 * t));
    const float da = half_bits_to_float(*reinterpret_cast<const uint16_t*>(pa));
    const float db = half_bits_to_float(*reinterpret_cast<const uint16_t*>(pb));
    const uint2 xb = tok_ok ? *reinterpret_cast<const uint2*>(xsm + g * xs_stride + blk * 32 + 8 * t)
                            : make_uint2(0u, 0u);
    uint32_t a[4] = {qa.x, qb.x, qa.y, qb.y};
    int cc[4] = {0, 0, 0, 0};
    mma_s8_16832(cc, a, xb.x, xb.y);
    const float2 x0 = ok0 ? dsm[s0 * nblk + blk] : make_float2(0.f, 0.f);
    const float2 x1 = ok1 ? dsm[s1 * nblk + blk] : make_float2(0.f, 0.f);
    acc[0] = fmaf(da * x0.x, i2f_exact22(cc[0]), acc[0]);
    acc[1] = fmaf(da * x1.x, i2f_exact22(cc[1]), acc[1]);
    acc[2] = fmaf(db * x0.x, i2f_exact22(cc[2]), acc[2]);
    acc[3] = fmaf(db * x1.x, i2f_exact22(cc[3]), acc[3]);
  }
#pragma unroll
  for (int q = 0; q < 4; q++) red[warp][lane][q] = acc[q];
  __syncthreads();
  if (warp != 0) return;
  float v[4];
#pragma unroll
  for (int q = 0; q < 4; q++) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) s += red[w][lane][q];
    v[q] = s;
  }
  const int r0 = tile * 16;
  if (epi == GE_SWIGLU) {
    const int o = (r0 >> 1) + g;  // 8-row interleaved gate/up blocks
    if (ok0) y[(int64_t)pr[s0] * ldy + o] = silu(v[0]) * v[2];
    if (ok1) y[(int64_t)pr[s1] * ldy + o] = silu(v[1]) * v[3];
  } else {
    if (ok0) { y[(int64_t)pr[s0] * ldy + r0 + g] = v[0]; y[(int64_t)pr[s0] * ldy + r0 + g + 8] = v[2]; }
    if (ok1) { y[(int64_t)pr[s1] * ldy + r0 + g] = v[1]; y[(int64_t)pr[s1] * ldy + r0 + g + 8] = v[3]; }
  }
  pdl_launch_dependents();
}

// combine: x[t] += sum_j w[t,j] * out[t*k + j] for pairs whose expert is local (others contribute 0)
__global__ void k_moe_combine(const float* __restrict__ out, int64_t ldo, const int* __restrict__ ids,
                              const float* __restrict__ wts, int k, int e0, int E_local, float* __restrict__ x,
                              int64_t ldx, int d) {
  pdl_wait();
  const int t = blockIdx.x;
  for (int i = threadIdx.x; i < d; i += blockDim.x) {
    float s = 0.f;
    for (int j = 0; j < k; j++) {
      const int e = ids[t * k + j] - e0;
      if (e >= 0 && e < E_local) s += wts[t * k + j] * out[((int64_t)t * k + j) * ldo + i];
    }
    x[(int64_t)t * ldx + i] += s;
  }
  pdl_launch_dependents();
}

cudaLaunchConfig_t cfg_pdl(dim3 g, dim3 b, size_t smem, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g;
  cfg.blockDim = b;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

void moe_route(torch::Tensor x, torch::Tensor gamma, double eps, torch::Tensor wr, int64_t k, bool norm_topk,
               torch::Tensor ids, torch::Tensor wts, c10::optional<torch::Tensor> rbias, int64_t kind) {
  TORCH_CHECK(kind == 0 || kind == 1, "route: kind 0 (softmax, top-k) or 1 (top-k, softmax)");
  const float* rb = nullptr;
  if (rbias.has_value()) {
    TORCH_CHECK(rbias->scalar_type() == torch::kFloat32 && rbias->numel() >= wr.size(0), "route: bias [E] f32");
    rb = rbias->data_ptr<float>();
  }
  const int T = (int)x.size(0), d = (int)x.size(1), E = (int)wr.size(0);
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.stride(1) == 1 && wr.size(1) == d && wr.is_contiguous(), "route");
  TORCH_CHECK(k >= 1 && k <= MAX_K && k <= E, "top-k");
  if (T == 0) return;
  cudaLaunchAttribute attr[1];
  const size_t smem = (size_t)(d + E) * 4;
  auto cfg = cfg_pdl(dim3(T), dim3(256), smem, attr);
  FAK_CUDA_CHECK(cudaFuncSetAttribute(k_moe_route, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_moe_route, (const float*)x.data_ptr<float>(), (int64_t)x.stride(0),
                                    (const float*)gamma.data_ptr<float>(), (float)eps, (const float*)wr.data_ptr<float>(),
                                    E, d, (int)k, (int)norm_topk, ids.data_ptr<int>(), wts.data_ptr<float>(), rb,
                                    (int)kind));
}

void moe_group(torch::Tensor ids, int64_t P, int64_t e0, int64_t E_local, int64_t max_chunks, torch::Tensor chunk_expert,
               torch::Tensor chunk_pairs, torch::Tensor n_chunks) {
  TORCH_CHECK(chunk_pairs.numel() >= max_chunks * CH && chunk_expert.numel() >= max_chunks, "chunk buffers");
  cudaLaunchAttribute attr[1];
  const size_t smem = (size_t)2 * E_local * 4;
  auto cfg = cfg_pdl(dim3(1), dim3(256), smem, attr);
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_moe_group, (const int*)ids.data_ptr<int>(), (int)P, (int)e0, (int)E_local,
                                    (int)max_chunks, chunk_expert.data_ptr<int>(), chunk_pairs.data_ptr<int>(),
                                    n_chunks.data_ptr<int>()));
}

void moe_qmmv(torch::Tensor w, int64_t qtype, int64_t rows_per_expert, int64_t K, int64_t pitch, torch::Tensor qx,
              torch::Tensor ds, int64_t topk, bool act_by_token, torch::Tensor chunk_expert, torch::Tensor chunk_pairs,
              torch::Tensor n_chunks, int64_t max_chunks, torch::Tensor y, int64_t epi, torch::Tensor err) {
  TORCH_CHECK(qtype == QT_Q8_0, "grouped expert GEMV: Q8_0 experts");
  TORCH_CHECK(K % 64 == 0 && rows_per_expert % 16 == 0 && pitch % 16 == 0, "shapes");
  TORCH_CHECK(y.scalar_type() == torch::kFloat32 && y.stride(1) == 1, "y");
  const size_t smem = (size_t)16 * pitch + (size_t)CH * (K + 32) + (size_t)CH * (K / 32) * 8;
  TORCH_CHECK(smem <= 220 * 1024, "tile too large");
  const int tiles = (int)(rows_per_expert / 16);
  cudaLaunchAttribute attr[1];
  auto cfg = cfg_pdl(dim3((unsigned)(max_chunks * tiles)), dim3(256), smem, attr);
  auto launch = [&](auto kern) {
    FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, (const uint8_t*)w.data_ptr<uint8_t>(), (int)rows_per_expert, (int)K,
                                      pitch, (const int8_t*)qx.data_ptr<int8_t>(),
                                      (const float2*)reinterpret_cast<float2*>(ds.data_ptr<float>()), (int)topk,
                                      (const int*)chunk_expert.data_ptr<int>(), (const int*)chunk_pairs.data_ptr<int>(),
                                      (const int*)n_chunks.data_ptr<int>(), y.data_ptr<float>(), (int64_t)y.stride(0),
                                      (int)epi, err.data_ptr<int>()));
  };
  if (act_by_token) launch(k_moe_qmmv_q8<1>);
  else launch(k_moe_qmmv_q8<0>);
}

void moe_combine(torch::Tensor out, torch::Tensor ids, torch::Tensor wts, int64_t k, int64_t e0, int64_t E_local,
                 torch::Tensor x) {
  const int T = (int)x.size(0), d = (int)x.size(1);
  if (T == 0) return;
  cudaLaunchAttribute attr[1];
  auto cfg = cfg_pdl(dim3(T), dim3(256), 0, attr);
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_moe_combine, (const float*)out.data_ptr<float>(), (int64_t)out.stride(0),
                                    (const int*)ids.data_ptr<int>(), (const float*)wts.data_ptr<float>(), (int)k,
                                    (int)e0, (int)E_local, x.data_ptr<float>(), (int64_t)x.stride(0), d));
}
