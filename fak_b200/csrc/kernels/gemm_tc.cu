// bf16 GEMM on the 5th-generation tensor cores: C[M, N] (op)= A[M, K] . B[N, K]^T (+ bias).
//
// A = activations (K-major), B = weights (K-major, the dequantized copy of a GGUF matrix).
// One CTA computes a 128 x BN tile; warp roles:
//   warp 0     TMA producer: 128 x 64 A box and BN x 64 B box per k-block (128-byte swizzle)
//              into a STAGES-deep shared-memory ring, completion tracked by mbarriers;
//   warp 1     allocates BN TMEM columns, then one thread issues tcgen05.mma (M=128, N=BN,
//              K=16 per instruction, 4 per k-block) and tcgen05.commit frees each stage;
//   warps 2-5  epilogue: tcgen05.ld the fp32 accumulator (warp w reads TMEM lanes
//              32*(w%4)..+31 = tile rows), fused bias / residual add / SwiGLU, global store.
// No TMA multicast is used, so the kernel is safe on multi-GPU runs.  The persistent variant
// (default) keeps two TMEM accumulators so each CTA's epilogue overlaps its next tile's MMAs.
//
// G_RS (persistent variant, tensor-parallel prefill): the reduce-scatter half of an all-reduce in
// the epilogue.  Output m-block mb belongs to rank mb % W; each fp32 tile is stored straight into
// the owner's peer buffer (slot [this rank][owner-local row][column]) and, once all 128 rows of the
// tile are written and fenced system-wide, a tile flag on the owner is released with the call's
// epoch.  The owner's k_p2p_rs_reduce then sums the W partials into the residual and broadcasts
// it, so the partials cross NVLink tile by tile while later tiles are still being computed.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cudaTypedefs.h>

#include <cstdlib>
#include <type_traits>

#include "mma.cuh"
#include "tc.cuh"

using namespace fak;

namespace {

constexpr int BM = 128;
constexpr int BK = 64;  // 64 bf16 = 128 bytes = one swizzle row
constexpr int GEMM_THREADS = 192;

enum GemmEpi : int { G_STORE = 0, G_ADD = 1, G_SWIGLU = 2, G_GEGLU = 3, G_RS = 4, G_OAI = 5 };
// the gated epilogues (8-column interleaved gate / up blocks); G_RS is not one of them
__host__ __device__ constexpr bool gated(int epi) { return epi == G_SWIGLU || epi == G_GEGLU || epi == G_OAI; }
// gated_out's code for a gated GEMM epilogue (the gpt-oss gate is 4 there)
__device__ __forceinline__ int gate_code(int epi) { return epi == G_OAI ? 4 : epi; }

constexpr int RS_MAX_W = 8;
struct RsPeers {
  uint8_t* base[RS_MAX_W];   // every rank's peer buffer
  int64_t parts_off;         // partial slots [W][MR][N] fp32
  int64_t flags_off;         // tile flags [m-block][n-block][RS_MAX_W] uint32
  int W, me, MR;             // ranks, this rank, owner-local rows per source slot
  uint32_t epoch;            // this call's flag value
};

FAK_DEV void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
FAK_DEV uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Sequence-parallel prefill: the A operand gathered from its owners (the all-gather fused into the
// GEMM's loads).  m-block mb of A lives in rank mb % W's shard at owner-local row (mb / W) * 128;
// map[r] is a TMA map over rank r's shard ([MR, K] bf16 in its peer buffer; plain tiled loads of
// peer memory, no multicast).  Before a tile's first load the producer waits (bounded) until the
// owner has released flags[mb] >= epoch in THIS rank's memory (owners push the flag to every rank).
struct alignas(64) AgMaps {
  CUtensorMap map[RS_MAX_W];
  const uint32_t* flags;   // local flags [m-block]
  uint32_t epoch;
  uint32_t spin;
  int W;
};

template <int BN, int STAGES>
struct GemmSmem {
  alignas(1024) __nv_bfloat16 a[STAGES][BM * BK];
  alignas(1024) __nv_bfloat16 b[STAGES][BN * BK];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t accum_full;
  uint32_t tmem_base;
};

template <typename OutT>
FAK_DEV void store_val(OutT* p, float v);
template <>
FAK_DEV void store_val<float>(float* p, float v) { *p = v; }
template <>
FAK_DEV void store_val<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <int BN, int STAGES, typename OutT>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
k_gemm_bf16(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b, int M, int N,
            int K, OutT* __restrict__ out, int64_t ldo, const float* __restrict__ bias, int epi, int* __restrict__ err,
            RsPeers rs, const __grid_constant__ AgMaps ag) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GemmSmem<BN, STAGES>& sm = *reinterpret_cast<GemmSmem<BN, STAGES>*>(base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * BM, n0 = blockIdx.y * BN;
  const int nkb = (K + BK - 1) / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      tc::mbar_init(&sm.full[s], 1);
      tc::mbar_init(&sm.empty[s], 1);
    }
    tc::mbar_init(&sm.accum_full, 1);
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmap_a);
    tc::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem_base, BN);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  // the A operand is produced by the previous kernel
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < nkb; kb++) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        tc::mbar_wait(&sm.empty[s], ph ^ 1, err);
        tc::mbar_arrive_expect_tx(&sm.full[s], (BM + BN) * BK * 2);
        tc::tma_load_2d(sm.a[s], &tmap_a, &sm.full[s], kb * BK, m0);
        tc::tma_load_2d(sm.b[s], &tmap_b, &sm.full[s], kb * BK, n0);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN);
      for (int kb = 0; kb < nkb; kb++) {
        const int s = kb % STAGES;
        const uint32_t ph = (kb / STAGES) & 1;
        tc::mbar_wait(&sm.full[s], ph, err);
        tc::tc_fence_after();
        const uint64_t ad = tc::smem_desc_sw128(sm.a[s]);
        const uint64_t bd = tc::smem_desc_sw128(sm.b[s]);
#pragma unroll
        for (int k = 0; k < BK / 16; k++) {
          // advance 16 bf16 = 32 bytes along K inside the swizzle row (encoded >> 4)
          tc::mma_bf16(tmem, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
        }
        tc::mma_commit(&sm.empty[s]);
      }
      tc::mma_commit(&sm.accum_full);
    }
  } else {
    // epilogue warps 2..5: TMEM lane quarter = warp % 4
    const int quarter = warp & 3;
    const int row = m0 + quarter * 32 + lane;
    tc::mbar_wait(&sm.accum_full, 0, err);
    tc::tc_fence_after();
    const uint32_t lane_addr = tmem + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
    for (int c = 0; c < BN; c += 16) {
      uint32_t r[16];
      tc::tmem_ld16(lane_addr + c, r);
      tc::tmem_ld_wait();
      if (row >= M) continue;
      const int col0 = n0 + c;
      if (gated(epi)) {
        // columns [col0, col0+8) are gate rows of outputs col0/2 + j, [col0+8, col0+16) the up rows
#pragma unroll
        for (int j = 0; j < 8; j++) {
          int col = col0 + j;
          if (col + 8 < N) {
            float g = __uint_as_float(r[j]), u = __uint_as_float(r[j + 8]);
            if (bias) { g += bias[col]; u += bias[col + 8]; }
            store_val(out + (int64_t)row * ldo + (col0 >> 1) + j, gated_out(gate_code(epi), g, u));
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < 16; j++) {
          int col = col0 + j;
          if (col < N) {
            float v = __uint_as_float(r[j]);
            if (bias) v += bias[col];
            OutT* p = out + (int64_t)row * ldo + col;
            if (epi == G_ADD) v += (float)*p;
            store_val(p, v);
          }
        }
      }
    }
  }
  pdl_launch_dependents();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, BN);
  }
}

// ---- persistent variant -----------------------------------------------------------------------
// One CTA per SM walks output tiles t = blockIdx.x, + gridDim.x, ... (m fastest, so the CTAs of a
// wave share weight column blocks through L2).  TMEM holds TWO 128 x BN fp32 accumulators (all 512
// columns at BN = 256): the MMA thread fills one while the epilogue warps drain the other, so the
// epilogue of tile i runs under the MMAs of tile i+1.  The producer streams k-blocks of successive
// tiles through the same smem ring without draining it between tiles.
template <int BN, int STAGES>
struct GemmSmemP {
  alignas(1024) __nv_bfloat16 a[STAGES][BM * BK];
  alignas(1024) __nv_bfloat16 b[STAGES][BN * BK];
  uint64_t full[STAGES];
  uint64_t empty[STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint32_t tmem_base;
};

template <typename OutT>
FAK_DEV void store16(OutT* p, const float (&v)[16], bool add, int n_valid);
template <>
FAK_DEV void store16<float>(float* p, const float (&v)[16], bool add, int n_valid) {
  if (n_valid == 16 && (reinterpret_cast<uintptr_t>(p) & 15) == 0) {
#pragma unroll
    for (int q = 0; q < 4; q++) {
      float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      if (add) {
        const float4 c = reinterpret_cast<const float4*>(p)[q];
        o.x += c.x; o.y += c.y; o.z += c.z; o.w += c.w;
      }
      reinterpret_cast<float4*>(p)[q] = o;
    }
    return;
  }
  for (int j = 0; j < n_valid; j++) p[j] = add ? p[j] + v[j] : v[j];
}
template <>
FAK_DEV void store16<__nv_bfloat16>(__nv_bfloat16* p, const float (&v)[16], bool add, int n_valid) {
  for (int j = 0; j < n_valid; j++) p[j] = __float2bfloat16_rn(add ? __bfloat162float(p[j]) + v[j] : v[j]);
}

template <int BN, int STAGES, typename OutT>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
k_gemm_bf16_persistent(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                       int M, int N, int K, OutT* __restrict__ out, int64_t ldo, const float* __restrict__ bias,
                       int epi, int* __restrict__ err, RsPeers rs, const __grid_constant__ AgMaps ag) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GemmSmemP<BN, STAGES>& sm = *reinterpret_cast<GemmSmemP<BN, STAGES>*>(base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nkb = (K + BK - 1) / BK;
  const int n_m = (M + BM - 1) / BM, n_n = (N + BN - 1) / BN;
  const int n_tiles = n_m * n_n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; s++) {
      tc::mbar_init(&sm.full[s], 1);
      tc::mbar_init(&sm.empty[s], 1);
    }
    for (int i = 0; i < 2; i++) {
      tc::mbar_init(&sm.acc_full[i], 1);
      tc::mbar_init(&sm.acc_empty[i], 4);  // one arrival per epilogue warp
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmap_a);
    tc::prefetch_tmap(&tmap_b);
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem_base, 2 * BN);
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_wait();

  if (warp == 0) {
    if (lane == 0) {
      int g = 0;  // k-blocks issued across tiles
      for (int r = 0; r < ag.W; r++) tc::prefetch_tmap(&ag.map[r]);
      for (int t = blockIdx.x; t < n_tiles; t += gridDim.x) {
        const int m0 = (t % n_m) * BM, n0 = (t / n_m) * BN;
        const CUtensorMap* amap = &tmap_a;
        int ay = m0;
        if (ag.W > 0) {   // gathered A: the owner's shard, once its rows are released
          const int mb = m0 / BM;
          amap = &ag.map[mb % ag.W];
          ay = (mb / ag.W) * BM;
          uint32_t it = 0;
          while (ld_acquire_sys_u32(ag.flags + mb) < ag.epoch) {
            if (++it > ag.spin) {
              report_error(err, 1);
              break;
            }
          }
        }
        for (int kb = 0; kb < nkb; kb++, g++) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          tc::mbar_wait(&sm.empty[s], ph ^ 1, err);
          tc::mbar_arrive_expect_tx(&sm.full[s], (BM + BN) * BK * 2);
          tc::tma_load_2d(sm.a[s], amap, &sm.full[s], kb * BK, ay);
          tc::tma_load_2d(sm.b[s], &tmap_b, &sm.full[s], kb * BK, n0);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = tc::idesc_bf16_f32(BM, BN);
      int g = 0, i = 0;
      for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, i++) {
        const int buf = i & 1, use = i >> 1;
        tc::mbar_wait(&sm.acc_empty[buf], (uint32_t)((use & 1) ^ 1), err);  // epilogue drained this buffer
        tc::tc_fence_after();
        const uint32_t acc = tmem + (uint32_t)(buf * BN);
        for (int kb = 0; kb < nkb; kb++, g++) {
          const int s = g % STAGES;
          const uint32_t ph = (g / STAGES) & 1;
          tc::mbar_wait(&sm.full[s], ph, err);
          tc::tc_fence_after();
          const uint64_t ad = tc::smem_desc_sw128(sm.a[s]);
          const uint64_t bd = tc::smem_desc_sw128(sm.b[s]);
#pragma unroll
          for (int k = 0; k < BK / 16; k++) tc::mma_bf16(acc, ad + 2 * k, bd + 2 * k, idesc, (kb | k) != 0);
          tc::mma_commit(&sm.empty[s]);
        }
        tc::mma_commit(&sm.acc_full[buf]);
      }
    }
  } else {
    const int quarter = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, i++) {
      const int buf = i & 1, use = i >> 1;
      const int m0 = (t % n_m) * BM, n0 = (t / n_m) * BN;
      const int row = m0 + quarter * 32 + lane;
      tc::mbar_wait(&sm.acc_full[buf], (uint32_t)(use & 1), err);
      tc::tc_fence_after();
      const uint32_t lane_addr = tmem + (uint32_t)(buf * BN) + ((uint32_t)(quarter * 32) << 16);
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        uint32_t r[16];
        tc::tmem_ld16(lane_addr + c, r);
        tc::tmem_ld_wait();
        const int col0 = n0 + c;
        if (row >= M || col0 >= N) continue;
        float v[16];
#pragma unroll
        for (int j = 0; j < 16; j++) v[j] = __uint_as_float(r[j]) + ((bias && col0 + j < N) ? bias[col0 + j] : 0.f);
        if (gated(epi)) {
          // columns [col0, col0+8) gate rows of outputs col0/2 + j, [col0+8, col0+16) the up rows
          float o[16];
#pragma unroll
          for (int j = 0; j < 8; j++) o[j] = gated_out(gate_code(epi), v[j], v[j + 8]);
          OutT* p = out + (int64_t)row * ldo + (col0 >> 1);
          if (col0 + 16 <= N && std::is_same<OutT, float>::value && ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
            float* pf = reinterpret_cast<float*>(p);
            reinterpret_cast<float4*>(pf)[0] = make_float4(o[0], o[1], o[2], o[3]);
            reinterpret_cast<float4*>(pf)[1] = make_float4(o[4], o[5], o[6], o[7]);
          } else if (col0 + 16 <= N && std::is_same<OutT, __nv_bfloat16>::value &&
                     ((reinterpret_cast<uintptr_t>(p) & 15) == 0)) {
            *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16(o[0], o[1]), pack_bf16(o[2], o[3]),
                                                      pack_bf16(o[4], o[5]), pack_bf16(o[6], o[7]));
          } else {
            for (int j = 0; j < 8; j++)
              if (col0 + j + 8 < N) store_val(p + j, o[j]);
          }
        } else if (epi == G_RS) {
          const int mb = m0 / BM;
          const int lr = (mb / rs.W) * BM + quarter * 32 + lane;   // row inside the owner's slot
          float* dst = reinterpret_cast<float*>(rs.base[mb % rs.W] + rs.parts_off) +
                       ((int64_t)rs.me * rs.MR + lr) * N + col0;
          store16<float>(dst, v, false, min(16, N - col0));
        } else {
          store16<OutT>(out + (int64_t)row * ldo + col0, v, epi == G_ADD, min(16, N - col0));
        }
      }
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sm.acc_empty[buf]);
      if (epi == G_RS) {
        // every row of the tile is in the owner's memory before its flag is released: the four
        // epilogue warps meet at a barrier, then ONE thread fences at system scope (cumulative over
        // the stores the barrier ordered before it) and releases the flag -- one system fence per
        // tile instead of one per thread
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (threadIdx.x == 64) {
          __threadfence_system();
          const int mb = m0 / BM, nb = n0 / BN, n_n = (N + BN - 1) / BN;
          uint32_t* f = reinterpret_cast<uint32_t*>(rs.base[mb % rs.W] + rs.flags_off) +
                        ((int64_t)mb * n_n + nb) * RS_MAX_W + rs.me;
          st_release_sys_u32(f, rs.epoch);
        }
      }
    }
  }
  pdl_launch_dependents();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 2 * BN);
  }
}

// ---- host: tensor maps through the driver entry point (no link-time libcuda dependency) ----
PFN_cuTensorMapEncodeTiled_v12000 get_encode() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    FAK_CUDA_CHECK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q));
    TORCH_CHECK(q == cudaDriverEntryPointSuccess && p, "cuTensorMapEncodeTiled unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

CUtensorMap make_map_bf16_kmajor(const void* ptr, int64_t rows, int64_t cols, int64_t ld_elems, int box_rows) {
  CUtensorMap m;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld_elems * 2};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = get_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  TORCH_CHECK(r == CUDA_SUCCESS, "cuTensorMapEncodeTiled failed: ", (int)r);
  return m;
}

template <int BN, int STAGES, typename OutT>
void launch_gemm(const torch::Tensor& a, const torch::Tensor& b, OutT* out, int64_t ldo, const float* bias, int epi,
                 int* err, bool persistent, const RsPeers& rs, const AgMaps& ag) {
  const int M = (int)a.size(0), K = (int)a.size(1), N = (int)b.size(0);
  CUtensorMap ma = make_map_bf16_kmajor(a.data_ptr(), M, K, a.stride(0), BM);
  CUtensorMap mb = make_map_bf16_kmajor(b.data_ptr(), N, K, b.stride(0), BN);
  const int tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  static int n_sm = 0;
  if (!n_sm) FAK_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, a.get_device()));
  size_t smem = persistent ? sizeof(GemmSmemP<BN, STAGES>) + 1024 : sizeof(GemmSmem<BN, STAGES>) + 1024;
  auto kern = persistent ? k_gemm_bf16_persistent<BN, STAGES, OutT> : k_gemm_bf16<BN, STAGES, OutT>;
  FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = persistent ? dim3((unsigned)std::min(tiles, n_sm)) : dim3((M + BM - 1) / BM, (N + BN - 1) / BN);
  cfg.blockDim = dim3(GEMM_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, ma, mb, M, N, K, out, ldo, bias, epi, err, rs, ag));
}

}  // namespace

// out (op)= a[M,K] . b[N,K]^T ; a, b bf16 K-major (row stride multiple of 8 elements, 16B-aligned base).
// epi: 0 store, 1 add into out, 2 SwiGLU over 8-column interleaved (gate x8, up x8) blocks -> out[:, N/2].
void gemm_bf16(torch::Tensor a, torch::Tensor b, torch::Tensor out, c10::optional<torch::Tensor> bias, int64_t epi,
               c10::optional<torch::Tensor> err) {
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == torch::kBFloat16 && a.dim() == 2 && a.stride(1) == 1, "a: [M,K] bf16");
  TORCH_CHECK(b.scalar_type() == torch::kBFloat16 && b.dim() == 2 && b.stride(1) == 1, "b: [N,K] bf16");
  TORCH_CHECK(a.size(1) == b.size(1), "K mismatch");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "row strides must be multiples of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              "operands must be 16-byte aligned");
  TORCH_CHECK(out.dim() == 2 && out.stride(1) == 1, "out: [M, *] row-major");
  const int64_t M = a.size(0), N = b.size(0);
  // epilogue codes as the GEMVs use them (4: the gpt-oss clamped gate, G_OAI here)
  TORCH_CHECK(epi >= 0 && epi <= 4, "gemm: epilogue");
  if (epi == 4) epi = G_OAI;
  TORCH_CHECK(out.size(0) >= M && out.size(1) >= (gated(epi) ? N / 2 : N), "out too small");
  if (gated(epi)) TORCH_CHECK(N % 16 == 0, "gated epilogues need 8-column interleaved gate/up blocks");
  if (M == 0 || N == 0) return;
  const float* bp = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() >= N, "bias");
    bp = bias->data_ptr<float>();
  }
  int* ep = err.has_value() ? err->data_ptr<int>() : nullptr;
  // persistent double-buffered-TMEM kernel by default; FAK_GEMM_PERSISTENT=0 selects one tile per CTA
  static const bool persistent = []() {
    const char* e = std::getenv("FAK_GEMM_PERSISTENT");
    return !(e && e[0] == '0');
  }();
  const RsPeers rs = {};
  static const AgMaps no_ag = {};
  if (out.scalar_type() == torch::kFloat32)
    launch_gemm<256, 4, float>(a, b, out.data_ptr<float>(), out.stride(0), bp, (int)epi, ep, persistent, rs, no_ag);
  else if (out.scalar_type() == torch::kBFloat16)
    launch_gemm<256, 4, __nv_bfloat16>(a, b, reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
                                        out.stride(0), bp, (int)epi, ep, persistent, rs, no_ag);
  else
    TORCH_CHECK(false, "out must be float32 or bfloat16");
}

// Tensor-parallel prefill: C = A . B^T with the reduce-scatter half of the all-reduce in the
// epilogue (G_RS above).  peers: int64 [W] base addresses of every rank's peer buffer; the owner
// rank of m-block mb is mb % W and holds MR rows per source slot (MR >= ceil(m-blocks / W) * 128).
// N must be a multiple of 4.  k_p2p_rs_reduce (p2p.cu) completes the all-reduce.
void gemm_bf16_rs(torch::Tensor a, torch::Tensor b, torch::Tensor peers, int64_t me, int64_t parts_off,
                  int64_t flags_off, int64_t MR, int64_t epoch, c10::optional<torch::Tensor> err) {
  TORCH_CHECK(a.is_cuda() && a.scalar_type() == torch::kBFloat16 && a.dim() == 2 && a.stride(1) == 1, "a: [M,K] bf16");
  TORCH_CHECK(b.scalar_type() == torch::kBFloat16 && b.dim() == 2 && b.stride(1) == 1, "b: [N,K] bf16");
  TORCH_CHECK(a.size(1) == b.size(1), "K mismatch");
  TORCH_CHECK(a.stride(0) % 8 == 0 && b.stride(0) % 8 == 0, "row strides must be multiples of 8 elements");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(a.data_ptr()) % 16 == 0 && reinterpret_cast<uintptr_t>(b.data_ptr()) % 16 == 0,
              "operands must be 16-byte aligned");
  TORCH_CHECK(peers.device().is_cpu() && peers.scalar_type() == torch::kInt64, "peers: int64 CPU tensor");
  const int W = (int)peers.numel();
  TORCH_CHECK(W >= 1 && W <= RS_MAX_W && me >= 0 && me < W, "gemm_bf16_rs: ranks");
  const int64_t M = a.size(0), N = b.size(0);
  TORCH_CHECK(N % 4 == 0 && parts_off % 16 == 0 && flags_off % 4 == 0, "gemm_bf16_rs: N % 4, offsets");
  const int64_t n_m = (M + BM - 1) / BM;
  TORCH_CHECK(MR >= (n_m + W - 1) / W * BM, "gemm_bf16_rs: MR too small for ", M, " rows over ", W, " ranks");
  if (M == 0 || N == 0) return;
  RsPeers rs = {};
  for (int r = 0; r < W; r++) rs.base[r] = reinterpret_cast<uint8_t*>(peers.data_ptr<int64_t>()[r]);
  rs.parts_off = parts_off;
  rs.flags_off = flags_off;
  rs.W = W;
  rs.me = (int)me;
  rs.MR = (int)MR;
  rs.epoch = (uint32_t)epoch;
  int* ep = err.has_value() ? err->data_ptr<int>() : nullptr;
  static const AgMaps no_ag = {};
  launch_gemm<256, 4, float>(a, b, nullptr, 0, nullptr, G_RS, ep, true, rs, no_ag);
}

// Sequence-parallel prefill GEMM: out (op)= A . B^T with A's m-blocks gathered from their owners'
// normalised shards (see AgMaps).  peers: int64 [W] peer-buffer bases; shard_off: the [MR, K] bf16
// shard in every buffer; flags_off: this rank's release flags [m-blocks]; M: rows of A and out.
void gemm_bf16_ag(int64_t M, torch::Tensor b, torch::Tensor out, torch::Tensor peers, int64_t me, int64_t shard_off,
                  int64_t MR, int64_t flags_off, int64_t epoch, int64_t spin, c10::optional<torch::Tensor> bias,
                  int64_t epi, c10::optional<torch::Tensor> err) {
  TORCH_CHECK(b.scalar_type() == torch::kBFloat16 && b.dim() == 2 && b.stride(1) == 1 && b.stride(0) % 8 == 0,
              "b: [N,K] bf16");
  TORCH_CHECK(peers.device().is_cpu() && peers.scalar_type() == torch::kInt64, "peers: int64 CPU tensor");
  const int W = (int)peers.numel();
  TORCH_CHECK(W >= 1 && W <= RS_MAX_W && me >= 0 && me < W, "gemm_bf16_ag: ranks");
  const int64_t N = b.size(0), K = b.size(1);
  TORCH_CHECK(K % 8 == 0 && shard_off % 16 == 0 && flags_off % 4 == 0, "gemm_bf16_ag: K % 8, offsets");
  TORCH_CHECK(MR >= ((M + BM - 1) / BM + W - 1) / W * BM, "gemm_bf16_ag: MR too small");
  if (epi == 4) epi = G_OAI;
  TORCH_CHECK((epi >= 0 && epi <= 3 || epi == G_OAI) && out.dim() == 2 && out.stride(1) == 1 && out.size(0) >= M &&
                  out.size(1) >= (gated(epi) ? N / 2 : N), "gemm_bf16_ag: out");
  if (M == 0 || N == 0) return;
  const float* bp = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() >= N, "bias");
    bp = bias->data_ptr<float>();
  }
  AgMaps ag = {};
  const int64_t* pp = peers.data_ptr<int64_t>();
  for (int r = 0; r < W; r++)
    ag.map[r] = make_map_bf16_kmajor(reinterpret_cast<const uint8_t*>(pp[r]) + shard_off, MR, K, K, BM);
  ag.flags = reinterpret_cast<const uint32_t*>(reinterpret_cast<const uint8_t*>(pp[me]) + flags_off);
  ag.epoch = (uint32_t)epoch;
  ag.spin = spin > 0 ? (uint32_t)spin : (1u << 26);
  ag.W = W;
  // launch_gemm takes M from a's rows and encodes a map of it for the plain path; in this mode that
  // map is never read (every A load goes through ag.map), so a view of this rank's shard stands in
  auto a_view = torch::from_blob(reinterpret_cast<uint8_t*>(pp[me]) + shard_off, {M, K},
                                 torch::TensorOptions().dtype(torch::kBFloat16).device(out.device()));
  const RsPeers rs = {};
  int* ep = err.has_value() ? err->data_ptr<int>() : nullptr;
  if (out.scalar_type() == torch::kFloat32)
    launch_gemm<256, 4, float>(a_view, b, out.data_ptr<float>(), out.stride(0), bp, (int)epi, ep, true, rs, ag);
  else if (out.scalar_type() == torch::kBFloat16)
    launch_gemm<256, 4, __nv_bfloat16>(a_view, b, reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
                                        out.stride(0), bp, (int)epi, ep, true, rs, ag);
  else
    TORCH_CHECK(false, "out must be float32 or bfloat16");
}
