// Quantized GEMV for decode: y[b, n] = sum_k W[n, k] * x[b, k] for a handful of tokens (B <= 8).
//
// W keeps its GGML block layout (Q4_K 144 B / Q6_K 210 B / Q8_0 34 B per block) with rows at a
// 16-byte-aligned pitch.  Activations arrive pre-quantized to int8 per 32-element block with a
// float2 (scale, exact float sum) per block, so every inner product is an integer dp4a:
//   Q4_K: sum (d*sc*q - dmin*m) * x  ~  d*sc*dx * sum(q*qx)  -  dmin*m * dx * sum(qx)
//   Q6_K: d*sc * dx * sum((q-32)*qx)         Q8_0: dw*dx * sum(qw*qx)
// (the reference's Q8 CUDA lane quantizes activations the same per-block way,
//  internal/compute/cuda_kernels.cu:374-427; its Q4_K lane keeps f32 activations, :478-526).
//
// Work split: one warp owns RW consecutive output rows; lane l walks the row in 64-weight
// "units" (u = l, l+32, ...), loading each unit's bytes for all RW rows with wide read-only
// loads, decoding them once into registers and reusing them for every token b.  Partial sums
// are reduced across the warp once at the end.  The epilogue fuses bias, residual add
// (y += acc, in place on the fp32 residual stream) or SwiGLU over interleaved (gate, up) rows.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "common.cuh"

using namespace fak;

namespace {

enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };

constexpr int GEMV_WARPS = 8;

struct XUnit {  // one token's 64 activations (two 32-blocks) for the current unit
  int w[16];
  float4 ds;  // (d0, s0, d1, s1)
};

FAK_DEV void load_x_unit(const int8_t* __restrict__ qx, const float2* __restrict__ ds, int64_t xoff0,
                         int64_t xoff1, int64_t blk0, int64_t blk1, XUnit& xu) {
  const int4* p0 = reinterpret_cast<const int4*>(qx + xoff0);
  const int4* p1 = reinterpret_cast<const int4*>(qx + xoff1);
  int4 a = __ldg(p0), b = __ldg(p0 + 1), c = __ldg(p1), d = __ldg(p1 + 1);
  xu.w[0] = a.x; xu.w[1] = a.y; xu.w[2] = a.z; xu.w[3] = a.w;
  xu.w[4] = b.x; xu.w[5] = b.y; xu.w[6] = b.z; xu.w[7] = b.w;
  xu.w[8] = c.x; xu.w[9] = c.y; xu.w[10] = c.z; xu.w[11] = c.w;
  xu.w[12] = d.x; xu.w[13] = d.y; xu.w[14] = d.z; xu.w[15] = d.w;
  float2 e = __ldg(ds + blk0), f = __ldg(ds + blk1);
  xu.ds = make_float4(e.x, e.y, f.x, f.y);
}

// ---------------------------------------------------------------------------------------------
// per-format unit decoders: produce 16 int8x4 words (elements of x-block 0 then x-block 1) and
// the float coefficients that multiply the integer dot products
// ---------------------------------------------------------------------------------------------
struct WUnitQ4K {
  uint32_t q[16];
  float ds0, ds1, mn0, mn1;  // d*sc, dmin*m for the two 32-blocks
};

FAK_DEV void load_q4k_unit(const uint8_t* __restrict__ row, int u, WUnitQ4K& wu) {
  int s = u >> 2, c = u & 3;
  const uint8_t* blk = row + (int64_t)s * 144;
  uint4 h = ldg_stream16(blk);
  uint4 q0 = ldg_stream16(blk + 16 + c * 32);
  uint4 q1 = ldg_stream16(blk + 32 + c * 32);
  float d = __half2float(__ushort_as_half((uint16_t)(h.x & 0xffff)));
  float dmin = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
  // scales bytes 0..11 live in h.y (0-3), h.z (4-7), h.w (8-11)
  int j0 = 2 * c, j1 = 2 * c + 1;
  auto byte_at = [&](int i) -> uint32_t {
    uint32_t w = i < 4 ? h.y : (i < 8 ? h.z : h.w);
    return (w >> (8 * (i & 3))) & 0xff;
  };
  uint32_t sc0, m0, sc1, m1;
  if (j0 < 4) {
    sc0 = byte_at(j0) & 63; m0 = byte_at(j0 + 4) & 63;
    sc1 = byte_at(j1) & 63; m1 = byte_at(j1 + 4) & 63;
  } else {
    sc0 = (byte_at(j0 + 4) & 15) | ((byte_at(j0 - 4) >> 6) << 4);
    m0 = (byte_at(j0 + 4) >> 4) | ((byte_at(j0) >> 6) << 4);
    sc1 = (byte_at(j1 + 4) & 15) | ((byte_at(j1 - 4) >> 6) << 4);
    m1 = (byte_at(j1 + 4) >> 4) | ((byte_at(j1) >> 6) << 4);
  }
  wu.ds0 = d * (float)sc0; wu.mn0 = dmin * (float)m0;
  wu.ds1 = d * (float)sc1; wu.mn1 = dmin * (float)m1;
  uint32_t raw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
  for (int i = 0; i < 8; i++) {
    wu.q[i] = raw[i] & 0x0F0F0F0Fu;
    wu.q[8 + i] = (raw[i] >> 4) & 0x0F0F0F0Fu;
  }
}

FAK_DEV float dot_q4k(const WUnitQ4K& wu, const XUnit& xu) {
  int s0 = 0, s1 = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    s0 = dp4a((int)wu.q[i], xu.w[i], s0);
    s1 = dp4a((int)wu.q[8 + i], xu.w[8 + i], s1);
  }
  return wu.ds0 * xu.ds.x * i2f_exact22(s0) + wu.ds1 * xu.ds.z * i2f_exact22(s1) - wu.mn0 * xu.ds.y - wu.mn1 * xu.ds.w;
}

struct WUnitQ8 {
  uint32_t q[16];
  float d0, d1;
};

FAK_DEV void load_q8_unit(const uint8_t* __restrict__ row, int u, WUnitQ8& wu) {
  const uint8_t* p = row + (int64_t)u * 68;  // two 34-byte blocks, 4-byte aligned
  uint32_t w[17];
#pragma unroll
  for (int i = 0; i < 17; i++) w[i] = ldg_stream4(p + 4 * i);
  wu.d0 = __half2float(__ushort_as_half((uint16_t)(w[0] & 0xffff)));
  wu.d1 = __half2float(__ushort_as_half((uint16_t)(w[8] >> 16)));
#pragma unroll
  for (int i = 0; i < 8; i++) wu.q[i] = __funnelshift_r(w[i], w[i + 1], 16);
#pragma unroll
  for (int i = 0; i < 8; i++) wu.q[8 + i] = w[9 + i];
}

FAK_DEV float dot_q8(const WUnitQ8& wu, const XUnit& xu) {
  int s0 = 0, s1 = 0;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    s0 = dp4a((int)wu.q[i], xu.w[i], s0);
    s1 = dp4a((int)wu.q[8 + i], xu.w[8 + i], s1);
  }
  return wu.d0 * xu.ds.x * i2f_exact22(s0) + wu.d1 * xu.ds.z * i2f_exact22(s1);
}

struct WUnitQ6K {
  uint32_t q[16];   // signed int8x4 (q-32): quarter p words 0..7, quarter p+2 words 8..15
  float sc[4];      // d*scale for elements [0,16) [16,32) of quarter p, then of quarter p+2
};

// read 4 bytes at a 2-byte-aligned address with aligned 4-byte loads
FAK_DEV uint32_t ld_u32_a2(const uint8_t* p) {
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint8_t* base = reinterpret_cast<const uint8_t*>(a & ~uintptr_t(3));
  uint32_t lo = ldg_stream4(base);
  if ((a & 3) == 0) return lo;
  uint32_t hi = ldg_stream4(base + 4);
  return __funnelshift_r(lo, hi, 16);
}

FAK_DEV void load_q6k_unit(const uint8_t* __restrict__ row, int u, WUnitQ6K& wu) {
  int s = u >> 2, c = u & 3, n = c >> 1, p = c & 1;
  const uint8_t* blk = row + (int64_t)s * 210;
  const uint8_t* ql = blk + n * 64 + p * 32;
  const uint8_t* qh = blk + 128 + n * 32;
  uint32_t l[8], h[8];
  uintptr_t a = reinterpret_cast<uintptr_t>(ql);
  if ((a & 3) == 0) {
#pragma unroll
    for (int i = 0; i < 8; i++) { l[i] = ldg_stream4(ql + 4 * i); h[i] = ldg_stream4(qh + 4 * i); }
  } else {
    const uint8_t* lb = ql - 2;
    const uint8_t* hb = qh - 2;
    uint32_t lw[9], hw[9];
#pragma unroll
    for (int i = 0; i < 9; i++) { lw[i] = ldg_stream4(lb + 4 * i); hw[i] = ldg_stream4(hb + 4 * i); }
#pragma unroll
    for (int i = 0; i < 8; i++) { l[i] = __funnelshift_r(lw[i], lw[i + 1], 16); h[i] = __funnelshift_r(hw[i], hw[i + 1], 16); }
  }
  uint32_t scw = ld_u32_a2(blk + 192 + 8 * n + 2 * p);      // scales sub 8n+2p, +1
  uint32_t scw2 = ld_u32_a2(blk + 192 + 8 * n + 2 * p + 4);  // scales sub 8n+2p+4, +5
  float d = __half2float(__ushort_as_half((uint16_t)(ld_u32_a2(blk + 208) & 0xffff)));
  wu.sc[0] = d * (float)(int8_t)(scw & 0xff);
  wu.sc[1] = d * (float)(int8_t)((scw >> 8) & 0xff);
  wu.sc[2] = d * (float)(int8_t)(scw2 & 0xff);
  wu.sc[3] = d * (float)(int8_t)((scw2 >> 8) & 0xff);
  int sh0 = 2 * p, sh1 = 2 * p + 4;
#pragma unroll
  for (int i = 0; i < 8; i++) {
    uint32_t q0 = (l[i] & 0x0F0F0F0Fu) | (((h[i] >> sh0) & 0x03030303u) << 4);
    uint32_t q1 = ((l[i] >> 4) & 0x0F0F0F0Fu) | (((h[i] >> sh1) & 0x03030303u) << 4);
    wu.q[i] = __vsub4(q0, 0x20202020u);
    wu.q[8 + i] = __vsub4(q1, 0x20202020u);
  }
}

FAK_DEV float dot_q6k(const WUnitQ6K& wu, const XUnit& xu) {
  int a0 = 0, a1 = 0, b0 = 0, b1 = 0;
#pragma unroll
  for (int i = 0; i < 4; i++) {
    a0 = dp4a((int)wu.q[i], xu.w[i], a0);
    a1 = dp4a((int)wu.q[4 + i], xu.w[4 + i], a1);
    b0 = dp4a((int)wu.q[8 + i], xu.w[8 + i], b0);
    b1 = dp4a((int)wu.q[12 + i], xu.w[12 + i], b1);
  }
  return xu.ds.x * (wu.sc[0] * i2f_exact22(a0) + wu.sc[1] * i2f_exact22(a1)) +
         xu.ds.z * (wu.sc[2] * i2f_exact22(b0) + wu.sc[3] * i2f_exact22(b1));
}

// x-block offsets (in elements, relative to the row start of x) of the two 32-blocks a unit covers
template <int QT>
FAK_DEV void unit_xblocks(int u, int& blk0, int& blk1) {
  if (QT == QT_Q6_K) {
    int s = u >> 2, c = u & 3, n = c >> 1, p = c & 1;
    blk0 = s * 8 + 4 * n + p;
    blk1 = blk0 + 2;
  } else {  // Q4_K (sub-blocks 2c, 2c+1) and Q8_0 (blocks 2u, 2u+1) are both consecutive
    blk0 = 2 * u;
    blk1 = 2 * u + 1;
  }
}

template <int QT>
struct WUnitOf;
template <> struct WUnitOf<QT_Q4_K> { using T = WUnitQ4K; };
template <> struct WUnitOf<QT_Q6_K> { using T = WUnitQ6K; };
template <> struct WUnitOf<QT_Q8_0> { using T = WUnitQ8; };

template <int QT>
FAK_DEV void load_unit(const uint8_t* row, int u, typename WUnitOf<QT>::T& wu) {
  if constexpr (QT == QT_Q4_K) load_q4k_unit(row, u, wu);
  else if constexpr (QT == QT_Q6_K) load_q6k_unit(row, u, wu);
  else load_q8_unit(row, u, wu);
}
template <int QT>
FAK_DEV float dot_unit(const typename WUnitOf<QT>::T& wu, const XUnit& xu) {
  if constexpr (QT == QT_Q4_K) return dot_q4k(wu, xu);
  else if constexpr (QT == QT_Q6_K) return dot_q6k(wu, xu);
  else return dot_q8(wu, xu);
}

template <int QT, int NB, int RW>
__global__ void __launch_bounds__(GEMV_WARPS * 32)
k_qgemv(const uint8_t* __restrict__ W, int N, int K, int64_t pitch, const int8_t* __restrict__ qx,
        const float2* __restrict__ ds, int B, float* __restrict__ y, int64_t ldy, const float* __restrict__ bias,
        int epi) {
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int row0 = (blockIdx.x * GEMV_WARPS + warp) * RW;
  const int n_units = K >> 6;
  const int64_t nblk_x = K >> 5;
  float acc[RW][NB];
#pragma unroll
  for (int r = 0; r < RW; r++)
#pragma unroll
    for (int b = 0; b < NB; b++) acc[r][b] = 0.f;

  // weights do not depend on the previous kernel: nothing to prefetch before the wait in this
  // simple form, but letting the launch overlap the predecessor's tail still hides launch latency
  pdl_wait();
  if (row0 < N) {
    for (int u = lane; u < n_units; u += 32) {
      typename WUnitOf<QT>::T wu[RW];
#pragma unroll
      for (int r = 0; r < RW; r++) {
        int row = min(row0 + r, N - 1);
        load_unit<QT>(W + (int64_t)row * pitch, u, wu[r]);
      }
      int blk0, blk1;
      unit_xblocks<QT>(u, blk0, blk1);
#pragma unroll
      for (int b = 0; b < NB; b++) {
        if (b < B) {
          XUnit xu;
          load_x_unit(qx, ds, b * (int64_t)K + blk0 * 32, b * (int64_t)K + blk1 * 32, b * nblk_x + blk0,
                      b * nblk_x + blk1, xu);
#pragma unroll
          for (int r = 0; r < RW; r++) acc[r][b] += dot_unit<QT>(wu[r], xu);
        }
      }
    }
  }
  pdl_launch_dependents();
#pragma unroll
  for (int r = 0; r < RW; r++)
#pragma unroll
    for (int b = 0; b < NB; b++) acc[r][b] = warp_sum(acc[r][b]);
  if (lane != 0 || row0 >= N) return;
  if (epi == EPI_SWIGLU) {
#pragma unroll
    for (int r = 0; r + 1 < RW; r += 2) {
      int row = row0 + r;
      if (row + 1 >= N) break;
#pragma unroll
      for (int b = 0; b < NB; b++) {
        if (b < B) {
          float g = acc[r][b], v = acc[r + 1][b];
          if (bias) { g += bias[row]; v += bias[row + 1]; }
          y[b * ldy + (row >> 1)] = silu(g) * v;
        }
      }
    }
    return;
  }
#pragma unroll
  for (int r = 0; r < RW; r++) {
    int row = row0 + r;
    if (row >= N) break;
    float bv = bias ? bias[row] : 0.f;
#pragma unroll
    for (int b = 0; b < NB; b++) {
      if (b < B) {
        float v = acc[r][b] + bv;
        if (epi == EPI_ADD) y[b * ldy + row] += v;
        else y[b * ldy + row] = v;
      }
    }
  }
}

template <int QT, int RW>
void launch_qgemv_rw(int NB, cudaLaunchConfig_t& cfg, const uint8_t* W, int N, int K, int64_t pitch,
                     const int8_t* qx, const float2* ds, int B, float* y, int64_t ldy, const float* bias, int epi) {
#define FAK_GEMV_CASE(nb)                                                                                \
  case nb:                                                                                               \
    FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_qgemv<QT, nb, RW>, W, N, K, pitch, qx, ds, B, y, ldy, bias, \
                                      epi));                                                             \
    break;
  switch (NB) {
    FAK_GEMV_CASE(1)
    FAK_GEMV_CASE(2)
    FAK_GEMV_CASE(3)
    FAK_GEMV_CASE(4)
    FAK_GEMV_CASE(5)
    FAK_GEMV_CASE(6)
    FAK_GEMV_CASE(7)
    FAK_GEMV_CASE(8)
    default:
      TORCH_CHECK(false, "qgemv: batch must be 1..8");
  }
#undef FAK_GEMV_CASE
}

}  // namespace

// y[B, N] (ldy) op= W[N, K] . x[B, K]; qx int8 [B, K], ds float [B, K/32, 2]
void qgemv(torch::Tensor w, int64_t qtype, int64_t N, int64_t K, int64_t pitch, torch::Tensor qx, torch::Tensor ds,
           int64_t B, torch::Tensor y, c10::optional<torch::Tensor> bias, int64_t epi) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kUInt8, "w: cuda uint8");
  TORCH_CHECK(K % 256 == 0 || (qtype == QT_Q8_0 && K % 64 == 0), "qgemv: K must be a multiple of 256 (64 for Q8_0)");
  TORCH_CHECK(pitch % 16 == 0, "qgemv: row pitch must be a multiple of 16 bytes");
  TORCH_CHECK(w.numel() >= N * pitch, "qgemv: weight buffer smaller than N*pitch");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0, "qgemv: weight base must be 16-byte aligned");
  TORCH_CHECK(qx.scalar_type() == torch::kInt8 && qx.is_contiguous() && qx.numel() >= B * K, "qgemv: qx");
  TORCH_CHECK(ds.scalar_type() == torch::kFloat32 && ds.is_contiguous() && ds.numel() >= B * K / 16, "qgemv: ds");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(qx.data_ptr()) % 16 == 0, "qgemv: qx must be 16-byte aligned");
  TORCH_CHECK(y.scalar_type() == torch::kFloat32 && y.dim() == 2 && y.stride(1) == 1, "qgemv: y must be [B, *] f32");
  TORCH_CHECK(B >= 1 && B <= 8, "qgemv: 1 <= B <= 8");
  int64_t out_cols = epi == EPI_SWIGLU ? N / 2 : N;
  TORCH_CHECK(y.size(0) >= B && y.size(1) >= out_cols, "qgemv: y too small");
  const float* bp = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() >= N, "qgemv: bias");
    bp = bias->data_ptr<float>();
  }
  TORCH_CHECK(epi != EPI_SWIGLU, "qgemv: the SwiGLU epilogue lives in qmmv (8-row interleaved gate/up tiles)");
  auto stream = at::cuda::getCurrentCUDAStream();
  // rows per warp: 4 when that still gives ~2 CTAs per SM, else 2
  int RW = (N / (4 * GEMV_WARPS) >= 296) ? 4 : 2;
  int grid = (int)((N + RW * GEMV_WARPS - 1) / (RW * GEMV_WARPS));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(GEMV_WARPS * 32);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const uint8_t* W = w.data_ptr<uint8_t>();
  const int8_t* q = qx.data_ptr<int8_t>();
  const float2* d2 = reinterpret_cast<const float2*>(ds.data_ptr<float>());
  float* yp = y.data_ptr<float>();
  int64_t ldy = y.stride(0);
  int nb = (int)B;
#define FAK_DISPATCH_QT(QTV)                                                                           \
  if (RW == 4) launch_qgemv_rw<QTV, 4>(nb, cfg, W, (int)N, (int)K, pitch, q, d2, nb, yp, ldy, bp, (int)epi); \
  else launch_qgemv_rw<QTV, 2>(nb, cfg, W, (int)N, (int)K, pitch, q, d2, nb, yp, ldy, bp, (int)epi);
  if (qtype == QT_Q4_K) { FAK_DISPATCH_QT(QT_Q4_K) }
  else if (qtype == QT_Q6_K) { FAK_DISPATCH_QT(QT_Q6_K) }
  else if (qtype == QT_Q8_0) { FAK_DISPATCH_QT(QT_Q8_0) }
  else TORCH_CHECK(false, "qgemv: unsupported qtype ", qtype);
#undef FAK_DISPATCH_QT
}
