// Shared device helpers for the sm_100a kernels.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>

#define FAK_DEV __device__ __forceinline__

namespace fak {

constexpr int QK_K = 256;
// QT_G4 is framework-internal: group-wise asymmetric 4-bit (AWQ / GPTQ) in 144-byte blocks of 256,
// [s0 f32][m0 f32][s1 f32][m1 f32][codes in the Q4_K nibble order], w = s_g * q - m_g per 128-group.
enum QType : int { QT_F32 = 0, QT_F16 = 1, QT_Q8_0 = 8, QT_Q4_K = 12, QT_Q6_K = 14, QT_BF16 = 30, QT_G4 = 64 };

FAK_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
FAK_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

FAK_DEV float half_bits_to_float(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// Little-endian unaligned reads from byte pointers (weights keep GGML block layout).
FAK_DEV uint16_t ld_u16(const uint8_t* p) { return (uint16_t)p[0] | ((uint16_t)p[1] << 8); }

// Streaming global loads for weights: read-only path, do not pollute L1.
FAK_DEV uint4 ldg_stream16(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
FAK_DEV uint32_t ldg_stream4(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
FAK_DEV uint2 ldg_stream8(const void* p) {
  uint2 r;
  asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}

// Programmatic dependent launch: let the next kernel in the stream start its
// independent prologue (weight prefetch) while this one drains, and wait for
// the previous kernel's results only where they are first read.
FAK_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
FAK_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Warm L2 with [base, base + bytes) for a LATER kernel (e.g. the next GEMV's weights while this
// kernel is latency-bound): CTA b issues the 64 KB pieces b, b + grid, ... from one thread; no
// shared memory is written and nothing waits for completion.  Call before pdl_wait: the bytes must
// not depend on the previous kernel.
FAK_DEV void l2_prefetch(const uint8_t* base, int64_t bytes) {
  if (base == nullptr || bytes <= 0 || threadIdx.x != 0) return;
  const int64_t nb = (int64_t)gridDim.x * gridDim.y * gridDim.z;
  const int64_t b = blockIdx.x + (int64_t)gridDim.x * (blockIdx.y + (int64_t)gridDim.y * blockIdx.z);
  constexpr int64_t CH = 65536;
  for (int64_t off = b * CH; off < bytes; off += nb * CH) {
    const uint32_t n = (uint32_t)(bytes - off < CH ? bytes - off : CH) & ~15u;
    if (n) asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + off), "r"(n) : "memory");
  }
}

FAK_DEV int dp4a(int a, int b, int c) { return __dp4a(a, b, c); }

// Exact int -> float for |c| < 2^22 without the (low-throughput) conversion pipe: adding c to
// the bit pattern of 1.5 * 2^23 gives the float 1.5 * 2^23 + c (one ulp = 1 in that binade), and
// subtracting 1.5 * 2^23 is exact.  Two full-rate ALU/FMA-pipe ops instead of one I2F.
FAK_DEV float i2f_exact22(int c) { return __int_as_float(c + 0x4B400000) - 12582912.0f; }

FAK_DEV float silu(float x) { return x / (1.0f + __expf(-x)); }
// GELU, tanh approximation (Hendrycks & Gimpel): 0.5 x (1 + tanh(sqrt(2/pi) (x + 0.044715 x^3)))
FAK_DEV float gelu_tanh(float x) { return 0.5f * x * (1.0f + tanhf(0.7978845608028654f * (x + 0.044715f * x * x * x))); }
// gated-FFN activation of the fused gate/up epilogues: 2 = SiLU (SwiGLU), 3 = GELU-tanh (GEGLU)
FAK_DEV float gated_act(int epi, float g) { return epi == 3 ? gelu_tanh(g) : silu(g); }

// Gated FFN output from a gate value g and an up value u.  epi: 2 SwiGLU, 3 GeGLU (GELU-tanh),
// 4 the gpt-oss clamped gate: (clamp(u, -7, 7) + 1) * g' * sigmoid(1.702 g') with g' = min(g, 7)
// (alpha 1.702 and limit 7 are the family's fixed constants; the loader refuses other values).
FAK_DEV float gated_out(int epi, float g, float u) {
  if (epi == 4) {
    g = fminf(g, 7.f);
    u = fminf(fmaxf(u, -7.f), 7.f);
    return (u + 1.f) * g / (1.f + expf(-1.702f * g));
  }
  return gated_act(epi, g) * u;
}

FAK_DEV float bf16_bits_lo(uint32_t v) { return __uint_as_float(v << 16); }
FAK_DEV float bf16_bits_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// Device-side error word: kernels never trap; they record a code and return.
// Codes: 1 = bounded wait expired, 2 = index out of range, 3 = bad argument, 4 = a peer rank never
// arrived at a fused all-reduce tile (tgemv epilogue).
// Programmatic dependent launch is requested on every launch of this library unless FAK_PDL=0.
// With it on, a profiler's span of a kernel includes its wait for the kernel before it, so a
// per-kernel attribution is taken with it off.
inline int pdl_allowed() {
  static const int on = [] {
    const char* e = getenv("FAK_PDL");
    return (e && e[0] == '0') ? 0 : 1;
  }();
  return on;
}

FAK_DEV void report_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// First-index argmax as one 64-bit key: order-preserving float bits in the high word, the
// complemented index in the low word, so the largest key is the largest value and, among equal
// values, the lowest index.  Key 0 stands for "no element".
FAK_DEV unsigned long long argmax_key(float v, uint32_t i) {
  uint32_t u = __float_as_uint(v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return ((unsigned long long)u << 32) | (unsigned long long)(0xFFFFFFFFu - i);
}
FAK_DEV int argmax_key_index(unsigned long long k) { return k ? (int)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0; }

// The largest key of x[i0, i1) for the calling CTA (valid in thread 0); index i is reported as
// i + id_off.  Every thread issues its PER loads (four floats each when VEC) before comparing, so
// a chunk costs one memory latency rather than one per element.
template <int PER, bool VEC>
FAK_DEV unsigned long long cta_best_key(const float* __restrict__ x, int i0, int i1, uint32_t id_off) {
  constexpr int E = VEC ? 4 : 1;
  float v[PER][E];
#pragma unroll
  for (int j = 0; j < PER; j++) {
    const int i = i0 + (j * (int)blockDim.x + (int)threadIdx.x) * E;
    if (VEC && i + 4 <= i1) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(x + i));
      v[j][0] = f.x;
      if constexpr (E == 4) { v[j][1] = f.y; v[j][2] = f.z; v[j][3] = f.w; }
    } else {
#pragma unroll
      for (int e = 0; e < E; e++) v[j][e] = i + e < i1 ? __ldg(x + i + e) : 0.f;
    }
  }
  unsigned long long best = 0ull;
#pragma unroll
  for (int j = 0; j < PER; j++) {
    const int i = i0 + (j * (int)blockDim.x + (int)threadIdx.x) * E;
#pragma unroll
    for (int e = 0; e < E; e++) {
      if (i + e < i1) {
        const unsigned long long k = argmax_key(v[j][e], (uint32_t)(i + e) + id_off);
        best = k > best ? k : best;
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long k = __shfl_xor_sync(0xffffffffu, best, o);
    best = k > best ? k : best;
  }
  __shared__ unsigned long long sk[32];
  if ((threadIdx.x & 31) == 0) sk[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0)
    for (int w = 1; w < (int)(blockDim.x >> 5); w++) best = sk[w] > best ? sk[w] : best;
  return best;
}

}  // namespace fak

#define FAK_CUDA_CHECK(expr)                                                                  \
  do {                                                                                        \
    cudaError_t _e = (expr);                                                                  \
    if (_e != cudaSuccess) {                                                                  \
      throw std::runtime_error(std::string("CUDA error: ") + cudaGetErrorString(_e) + " at " + \
                               __FILE__ + ":" + std::to_string(__LINE__));                    \
    }                                                                                         \
  } while (0)
