// Block quantizers / dequantizers for the GGML formats kept resident on the GPU,
// plus the int8 activation quantizer that feeds the dp4a GEMV.
//
// Quantizers reproduce fak_b200/gguf/quants.py step for step in IEEE float32
// (no contraction into FMA: products use __fmul_rn) so GPU-built checkpoints
// are byte-identical to CPU-built ones.  Dequantizers follow the GGML layouts
// (reference decoders: internal/ggufload/gguf_dequant.go:709 Q4_K, :803 Q6_K, :793 Q8_0).
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "common.cuh"

using namespace fak;

namespace {

// ------------------------------------------------------------------------------------------
// quantizers (one thread per block)
// ------------------------------------------------------------------------------------------
__global__ void k_quantize_q8_0(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t nblocks) {
  int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * 32;
  float amax = 0.f;
  for (int i = 0; i < 32; i++) amax = fmaxf(amax, fabsf(xb[i]));
  __half d = __float2half_rn(amax / 127.0f);
  float df = __half2float(d);
  uint8_t* o = out + b * 34;
  *reinterpret_cast<uint16_t*>(o) = __half_as_ushort(d);  // blocks are 34 B: 2-byte aligned
  for (int i = 0; i < 32; i++) {
    float q = df == 0.f ? 0.f : rintf(xb[i] / df);
    q = fminf(fmaxf(q, -127.f), 127.f);
    o[2 + i] = (uint8_t)(int8_t)q;
  }
}

__global__ void k_quantize_q4_k(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t nblocks) {
  int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * QK_K;
  float scale[8], mins[8];
  float smax = 0.f, mmax = 0.f;
  for (int j = 0; j < 8; j++) {
    float mn = xb[j * 32], mx = xb[j * 32];
    for (int i = 1; i < 32; i++) {
      mn = fminf(mn, xb[j * 32 + i]);
      mx = fmaxf(mx, xb[j * 32 + i]);
    }
    mn = fminf(mn, 0.f);
    scale[j] = (mx - mn) / 15.0f;
    mins[j] = -mn;
    smax = fmaxf(smax, scale[j]);
    mmax = fmaxf(mmax, mins[j]);
  }
  __half d = __float2half_rn(smax / 63.0f);
  __half dmin = __float2half_rn(mmax / 63.0f);
  float df = __half2float(d), dmf = __half2float(dmin);
  int sc[8], m[8];
  for (int j = 0; j < 8; j++) {
    float s = df > 0.f ? rintf(scale[j] / df) : 0.f;
    float mm = dmf > 0.f ? rintf(mins[j] / dmf) : 0.f;
    sc[j] = (int)fminf(fmaxf(s, 0.f), 63.f);
    m[j] = (int)fminf(fmaxf(mm, 0.f), 63.f);
  }
  uint8_t* o = out + b * 144;
  *reinterpret_cast<uint32_t*>(o) = (uint32_t)__half_as_ushort(d) | ((uint32_t)__half_as_ushort(dmin) << 16);
  for (int j = 0; j < 4; j++) {
    o[4 + j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    o[8 + j] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
    o[12 + j] = (uint8_t)((sc[j + 4] & 0x0f) | ((m[j + 4] & 0x0f) << 4));
  }
  for (int c = 0; c < 4; c++) {
    float es0 = __fmul_rn(df, (float)sc[2 * c]), em0 = __fmul_rn(dmf, (float)m[2 * c]);
    float es1 = __fmul_rn(df, (float)sc[2 * c + 1]), em1 = __fmul_rn(dmf, (float)m[2 * c + 1]);
    for (int l = 0; l < 32; l++) {
      float q0 = es0 > 0.f ? rintf(__fadd_rn(xb[c * 64 + l], em0) / es0) : 0.f;
      float q1 = es1 > 0.f ? rintf(__fadd_rn(xb[c * 64 + 32 + l], em1) / es1) : 0.f;
      int i0 = (int)fminf(fmaxf(q0, 0.f), 15.f), i1 = (int)fminf(fmaxf(q1, 0.f), 15.f);
      o[16 + c * 32 + l] = (uint8_t)(i0 | (i1 << 4));
    }
  }
}

__global__ void k_quantize_q6_k(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t nblocks) {
  int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * QK_K;
  float scale[16];
  float amax_s = 0.f;
  for (int j = 0; j < 16; j++) {
    int idx = 0;
    float best = fabsf(xb[j * 16]);
    for (int i = 1; i < 16; i++) {
      float a = fabsf(xb[j * 16 + i]);
      if (a > best) { best = a; idx = i; }
    }
    scale[j] = xb[j * 16 + idx] / -32.0f;
    amax_s = fmaxf(amax_s, fabsf(scale[j]));
  }
  __half d = __float2half_rn(amax_s / 127.0f);
  float df = __half2float(d);
  int sc[16];
  for (int j = 0; j < 16; j++) {
    float s = df > 0.f ? rintf(scale[j] / df) : 0.f;
    sc[j] = (int)fminf(fmaxf(s, -128.f), 127.f);
  }
  uint8_t* o = out + b * 210;
  uint8_t q[256];
  for (int j = 0; j < 16; j++) {
    float eff = __fmul_rn(df, (float)sc[j]);
    for (int i = 0; i < 16; i++) {
      float v = eff != 0.f ? rintf(xb[j * 16 + i] / eff) : 0.f;
      q[j * 16 + i] = (uint8_t)((int)fminf(fmaxf(v, -32.f), 31.f) + 32);
    }
  }
  for (int n = 0; n < 2; n++) {
    for (int l = 0; l < 32; l++) {
      int q0 = q[n * 128 + l], q1 = q[n * 128 + 32 + l], q2 = q[n * 128 + 64 + l], q3 = q[n * 128 + 96 + l];
      o[n * 64 + l] = (uint8_t)((q0 & 15) | ((q2 & 15) << 4));
      o[n * 64 + 32 + l] = (uint8_t)((q1 & 15) | ((q3 & 15) << 4));
      o[128 + n * 32 + l] = (uint8_t)((q0 >> 4) | ((q1 >> 4) << 2) | ((q2 >> 4) << 4) | ((q3 >> 4) << 6));
    }
  }
  for (int j = 0; j < 16; j++) o[192 + j] = (uint8_t)(int8_t)sc[j];
  *reinterpret_cast<uint16_t*>(o + 208) = __half_as_ushort(d);  // 210*b + 208 is even
}

// G4: one thread per 256-weight block (two 128-groups); scale (max - min) / 15 with min <= 0 <= max,
// zero point rint(-min / s), codes clamp(rint(x / s) + z, 0, 15) -- the numpy codec's arithmetic.
__global__ void k_quantize_g4(const float* __restrict__ x, uint8_t* __restrict__ out, int64_t nblocks) {
  int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float* xb = x + b * QK_K;
  uint8_t* ob = out + b * 144;
  float hdr[4];
  for (int g = 0; g < 2; g++) {
    float lo = 0.f, hi = 0.f;
    for (int i = 0; i < 128; i++) {
      lo = fminf(lo, xb[128 * g + i]);
      hi = fmaxf(hi, xb[128 * g + i]);
    }
    float s = (hi - lo) / 15.0f;
    if (!(s > 0.f)) s = 1.0f;
    const float z = fminf(fmaxf(rintf(-lo / s), 0.f), 15.f);
    hdr[2 * g] = s;
    hdr[2 * g + 1] = z * s;
    for (int i = 0; i < 128; i += 64) {
      for (int l = 0; l < 32; l++) {
        const int e = 128 * g + i + l;
        const int q0 = (int)fminf(fmaxf(rintf(xb[e] / s) + z, 0.f), 15.f);
        const int q1 = (int)fminf(fmaxf(rintf(xb[e + 32] / s) + z, 0.f), 15.f);
        ob[16 + (e / 64) * 32 + l] = (uint8_t)(q0 | (q1 << 4));
      }
    }
  }
  for (int k = 0; k < 4; k++) reinterpret_cast<float*>(ob)[k] = hdr[k];
}

// ------------------------------------------------------------------------------------------
// dequantizers: rows of GGML blocks (row pitch in bytes may exceed the packed row) -> T
// one thread per 32 output elements
// ------------------------------------------------------------------------------------------
template <typename T>
FAK_DEV void store_out(T* p, float v);
template <>
FAK_DEV void store_out<float>(float* p, float v) { *p = v; }
template <>
FAK_DEV void store_out<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T>
__global__ void k_dequant(const uint8_t* __restrict__ w, int qtype, int64_t rows, int64_t cols, int64_t pitch,
                          T* __restrict__ out) {
  int64_t g = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // group of 32 elements
  int64_t groups_per_row = cols / 32;
  if (g >= rows * groups_per_row) return;
  int64_t r = g / groups_per_row;
  int64_t c0 = (g % groups_per_row) * 32;
  const uint8_t* row = w + r * pitch;
  T* o = out + r * cols + c0;
  if (qtype == QT_Q8_0) {
    const uint8_t* blk = row + (c0 / 32) * 34;
    float d = half_bits_to_float(ld_u16(blk));
    for (int i = 0; i < 32; i++) store_out(o + i, d * (float)(int8_t)blk[2 + i]);
  } else if (qtype == QT_Q4_K) {
    int64_t sb = c0 / QK_K;
    int j = (int)((c0 % QK_K) / 32);  // sub-block 0..7
    const uint8_t* blk = row + sb * 144;
    float d = half_bits_to_float(ld_u16(blk)), dmin = half_bits_to_float(ld_u16(blk + 2));
    const uint8_t* s = blk + 4;
    int sc, m;
    if (j < 4) {
      sc = s[j] & 63; m = s[j + 4] & 63;
    } else {
      sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
      m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
    float d1 = d * (float)sc, m1 = dmin * (float)m;
    const uint8_t* q = blk + 16 + (j / 2) * 32;
    int shift = (j & 1) * 4;
    for (int l = 0; l < 32; l++) store_out(o + l, d1 * (float)((q[l] >> shift) & 15) - m1);
  } else if (qtype == QT_G4) {
    int64_t sb = c0 / QK_K;
    int j = (int)((c0 % QK_K) / 32);  // sub-block 0..7; groups of 128 = sub-blocks 0-3 / 4-7
    const uint8_t* blk = row + sb * 144;
    const float sc = reinterpret_cast<const float*>(blk)[2 * (j >> 2)];
    const float mn = reinterpret_cast<const float*>(blk)[2 * (j >> 2) + 1];
    const uint8_t* q = blk + 16 + (j / 2) * 32;
    int shift = (j & 1) * 4;
    for (int l = 0; l < 32; l++) store_out(o + l, sc * (float)((q[l] >> shift) & 15) - mn);
  } else if (qtype == QT_Q6_K) {
    int64_t sb = c0 / QK_K;
    int e0 = (int)(c0 % QK_K);  // multiple of 32
    const uint8_t* blk = row + sb * 210;
    float d = half_bits_to_float(ld_u16(blk + 208));
    int n = e0 / 128, k = (e0 % 128) / 32;  // quarter within the half
    const uint8_t* ql = blk + n * 64 + (k & 1) * 32;
    const uint8_t* qh = blk + 128 + n * 32;
    int lshift = (k >> 1) * 4, hshift = k * 2;
    for (int l = 0; l < 32; l++) {
      int q = ((ql[l] >> lshift) & 15) | (((qh[l] >> hshift) & 3) << 4);
      int sub = (e0 + l) / 16;
      float sc = (float)(int8_t)blk[192 + sub];
      store_out(o + l, d * sc * (float)(q - 32));
    }
  } else if (qtype == QT_F32) {
    const float* src = reinterpret_cast<const float*>(row) + c0;
    for (int i = 0; i < 32; i++) store_out(o + i, src[i]);
  } else if (qtype == QT_F16) {
    const __half* src = reinterpret_cast<const __half*>(row) + c0;
    for (int i = 0; i < 32; i++) store_out(o + i, __half2float(src[i]));
  } else if (qtype == QT_BF16) {
    const __nv_bfloat16* src = reinterpret_cast<const __nv_bfloat16*>(row) + c0;
    for (int i = 0; i < 32; i++) store_out(o + i, __bfloat162float(src[i]));
  }
}

// ------------------------------------------------------------------------------------------
// activation quantizer: x [B,K] fp32 -> qx int8 [B,K], ds float2 [B,K/32] = (scale, scale * sum(qx)):
// the offset term of K-quant / G4 weights then uses the same quantized values as the dot product
// (an exact-sum offset with quantized products nearly doubles the rounding error of offset formats)
// optional fused RMSNorm (gamma != nullptr).  One CTA per row, 256 threads.
// ------------------------------------------------------------------------------------------
__global__ void k_quant_act(const float* __restrict__ x, int64_t ldx, const float* __restrict__ gamma, float eps,
                            int K, int8_t* __restrict__ qx, float2* __restrict__ ds) {
  pdl_wait();
  int b = blockIdx.x;
  const float* xr = x + b * ldx;
  __shared__ float red[8];
  float inv = 1.f;
  if (gamma) {
    float ss = 0.f;
    for (int i = threadIdx.x; i < K; i += blockDim.x) ss += xr[i] * xr[i];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      v = warp_sum(v);
      if (threadIdx.x == 0) red[0] = v;
    }
    __syncthreads();
    inv = rsqrtf(red[0] / (float)K + eps);
  }
  pdl_launch_dependents();
  int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  for (int blk = warp; blk < K / 32; blk += nw) {
    int i = blk * 32 + lane;
    float v = xr[i] * inv;
    if (gamma) v *= gamma[i];
    float amax = warp_max(fabsf(v));
    float d = amax / 127.f;
    float q = d > 0.f ? rintf(v / d) : 0.f;
    float s = warp_sum(q) * d;  // sum of the dequantized values (exact integer sum x scale)
    qx[(int64_t)b * K + i] = (int8_t)q;
    if (lane == 0) ds[(int64_t)b * (K / 32) + blk] = make_float2(d, s);
  }
}

}  // namespace

// ------------------------------------------------------------------------------------------
// host entry points
// ------------------------------------------------------------------------------------------
torch::Tensor quantize_blocks(torch::Tensor x, int64_t qtype) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.is_contiguous(), "x: contiguous cuda f32");
  int64_t n = x.numel();
  int64_t blk = qtype == QT_Q8_0 ? 32 : 256;
  int64_t bytes = qtype == QT_Q8_0 ? 34 : ((qtype == QT_Q4_K || qtype == QT_G4) ? 144 : 210);
  TORCH_CHECK(qtype == QT_Q8_0 || qtype == QT_Q4_K || qtype == QT_Q6_K || qtype == QT_G4, "unsupported qtype");
  TORCH_CHECK(n % blk == 0, "element count not a multiple of the block size");
  int64_t nb = n / blk;
  auto out = torch::empty({nb * bytes}, x.options().dtype(torch::kUInt8));
  auto stream = at::cuda::getCurrentCUDAStream();
  int threads = 128;
  int64_t grid = (nb + threads - 1) / threads;
  if (nb == 0) return out;
  if (qtype == QT_Q8_0)
    k_quantize_q8_0<<<grid, threads, 0, stream>>>(x.data_ptr<float>(), out.data_ptr<uint8_t>(), nb);
  else if (qtype == QT_Q4_K)
    k_quantize_q4_k<<<grid, threads, 0, stream>>>(x.data_ptr<float>(), out.data_ptr<uint8_t>(), nb);
  else if (qtype == QT_G4)
    k_quantize_g4<<<grid, threads, 0, stream>>>(x.data_ptr<float>(), out.data_ptr<uint8_t>(), nb);
  else
    k_quantize_q6_k<<<grid, threads, 0, stream>>>(x.data_ptr<float>(), out.data_ptr<uint8_t>(), nb);
  FAK_CUDA_CHECK(cudaGetLastError());
  return out;
}

torch::Tensor dequantize_rows(torch::Tensor w, int64_t qtype, int64_t rows, int64_t cols, int64_t pitch,
                              c10::ScalarType out_dtype) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kUInt8, "w: cuda uint8");
  TORCH_CHECK(cols % 32 == 0, "cols must be a multiple of 32");
  TORCH_CHECK(w.numel() >= rows * pitch, "weight buffer too small for rows*pitch");
  auto out = torch::empty({rows, cols}, w.options().dtype(out_dtype));
  int64_t groups = rows * (cols / 32);
  if (groups == 0) return out;
  int threads = 256;
  int64_t grid = (groups + threads - 1) / threads;
  auto stream = at::cuda::getCurrentCUDAStream();
  if (out_dtype == torch::kFloat32)
    k_dequant<float><<<grid, threads, 0, stream>>>(w.data_ptr<uint8_t>(), (int)qtype, rows, cols, pitch,
                                                   out.data_ptr<float>());
  else if (out_dtype == torch::kBFloat16)
    k_dequant<__nv_bfloat16><<<grid, threads, 0, stream>>>(w.data_ptr<uint8_t>(), (int)qtype, rows, cols, pitch,
                                                            reinterpret_cast<__nv_bfloat16*>(out.data_ptr()));
  else
    TORCH_CHECK(false, "dequantize_rows: out dtype must be float32 or bfloat16");
  FAK_CUDA_CHECK(cudaGetLastError());
  return out;
}

void quant_act(torch::Tensor x, c10::optional<torch::Tensor> gamma, double eps, torch::Tensor qx, torch::Tensor ds) {
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.dim() == 2 && x.stride(1) == 1, "x: [B,K] f32");
  int B = (int)x.size(0), K = (int)x.size(1);
  TORCH_CHECK(K % 32 == 0, "K must be a multiple of 32");
  TORCH_CHECK(qx.scalar_type() == torch::kInt8 && qx.is_contiguous() && qx.numel() >= (int64_t)B * K, "qx");
  TORCH_CHECK(ds.scalar_type() == torch::kFloat32 && ds.is_contiguous() && ds.numel() >= (int64_t)B * K / 16, "ds");
  const float* g = nullptr;
  if (gamma.has_value()) {
    TORCH_CHECK(gamma->scalar_type() == torch::kFloat32 && gamma->numel() == K, "gamma");
    g = gamma->data_ptr<float>();
  }
  if (B == 0) return;
  auto stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B);
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_quant_act, (const float*)x.data_ptr<float>(), (int64_t)x.stride(0), g,
                                    (float)eps, K, qx.data_ptr<int8_t>(), reinterpret_cast<float2*>(ds.data_ptr<float>())));
}
