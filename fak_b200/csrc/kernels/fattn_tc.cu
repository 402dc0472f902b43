// Prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), over the paged KV cache.
//
// One CTA per (128-query tile of one sequence, query head).  The chunk's queries attend causally to
// the sequence's cached prefix and to themselves (their K/V are already in the pages).  Warp roles:
//   warp 0      TMA producer: the Q tile once (two 64-column halves, 128-byte swizzle), then per KV
//               tile of 128 keys the 8 pages of K (one stage, refilled as soon as S of the previous
//               tile is done) and of V (two stages) as 16 x 64 boxes of a 3-D map over the cache,
//               [layer * pages * kv heads, 16 tokens, head dim];
//   warp 1      one thread issues tcgen05.mma: S_j = Q K_j^T (M = N = 128, K = head dim) into one of
//               two TMEM S buffers, and O += P_j V_j (V as an MN-major operand: keys x head dim as it
//               sits in the pages) into one TMEM O buffer that lives for the whole CTA;
//   warps 2-9   softmax, two threads per query row (TMEM lane = row; warps w and w + 4 cover the
//               same lane quarter): warps 2-5 take keys 0-63 of each tile, warps 6-9 keys 64-127.
//               Each reads its half row of S once into registers (the S buffer is then free), the
//               two halves exchange their row max through shared memory (a named barrier per lane
//               quarter), and each writes its half of P = 2^(S - m) as bf16 into shared memory in
//               the 128-byte-swizzled K-major layout the P.V MMA reads.  The exponent base m is the
//               running row max, moved only when it grew by more than 2^8 (then each half rescales
//               its 64 columns of the rows' O in TMEM, once the previous P.V has completed), so
//               P <= 256 and most tiles touch O not at all; the halves' row sums add at the end.
// P has two buffers, so the softmax of tile j + 1 does not wait for P.V_j (only an O rescale does),
// and S of tile j + 1 is computed while tile j's softmax runs.  Every wait is bounded (tc::mbar_wait);
// no load uses multicast.  Head dim 128, no window / soft-cap (those shapes use k_prefill_attn).
// Reference: k_flash_attention, internal/compute/cuda_kernels.cu:701-759 (one block per head, SIMT).
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>
#include <cudaTypedefs.h>

#include "mma.cuh"
#include "tc.cuh"

using namespace fak;

namespace {

constexpr int FA_QT = 128;     // queries per tile
constexpr int FA_KT = 128;     // keys per KV tile (8 pages)
constexpr int FA_D = 128;      // head dim
constexpr int FA_PG = 16;      // tokens per page
constexpr int FA_STAGES = 2;
constexpr int FA_THREADS = 320;   // producer, MMA issuer, 8 softmax warps
constexpr float FA_HEADROOM = 8.f;   // log2 growth of a row max tolerated before O is rescaled

struct FaSmem {
  alignas(1024) __nv_bfloat16 q[2][FA_QT * 64];               // [D half][128 rows x 64]
  alignas(1024) __nv_bfloat16 k[2][FA_KT * 64];               // one stage: [D half][128 keys x 64]
  alignas(1024) __nv_bfloat16 v[FA_STAGES][2][FA_KT * 64];    // [stage][D half][128 keys x 64]
  alignas(1024) __nv_bfloat16 p[2][2][FA_QT * 64];            // [buffer][key half][128 rows x 64 keys]
  uint64_t q_full;
  uint64_t k_full, k_empty;
  uint64_t v_full[FA_STAGES], v_empty[FA_STAGES];
  uint64_t s_full[2], s_free[2];
  uint64_t p_full[2], p_free[2];   // per P buffer: written by the softmax / read by its P.V (done)
  float red[2][2][FA_QT];   // row max of each key half, by tile parity
  float lsum[2][FA_QT];     // row sums of each key half (end of the CTA)
  uint32_t tmem_base;
};

FAK_DEV void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          tc::smem_addr(dst)),
      "l"(map), "r"(tc::smem_addr(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// the hardware base-2 exponential (flushes denormal results to zero; 2^-inf = 0)
FAK_DEV float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Shared-memory descriptor of an MN-major operand in the 128-byte swizzle (rows of 128 bytes along
// MN = 64 bf16, atoms of 8 such rows along K): SBO = byte step between 8-row groups along K, LBO =
// byte step between 64-element groups along MN.
FAK_DEV uint64_t smem_desc_sw128_mn(const void* p, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t addr = tc::smem_addr(p);
  uint64_t d = 0;
  d |= (addr & 0x3FFFFull) >> 4;
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;   // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;   // 128-byte swizzle
  return d;
}

__global__ void __launch_bounds__(FA_THREADS, 1)
k_prefill_attn_tc(const __grid_constant__ CUtensorMap tmap_q, const __grid_constant__ CUtensorMap tmap_k,
                  const __grid_constant__ CUtensorMap tmap_v, int layer, int n_pages, int Hkv, int Hq,
                  const int* __restrict__ block_table, int bt_stride, const int* __restrict__ tile_seq,
                  const int* __restrict__ tile_q0, const int* __restrict__ seq_qoff, const int* __restrict__ seq_qlen,
                  const int* __restrict__ seq_pos0, __nv_bfloat16* __restrict__ out, int64_t ldo, float scale_log2,
                  int* __restrict__ err) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  FaSmem& sm = *reinterpret_cast<FaSmem*>(base);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile = blockIdx.x, h = blockIdx.y;
  const int g = h / (Hq / Hkv);

  if (threadIdx.x == 0) {
    tc::mbar_init(&sm.q_full, 1);
    tc::mbar_init(&sm.k_full, 1);
    tc::mbar_init(&sm.k_empty, 1);
    for (int s = 0; s < FA_STAGES; s++) {
      tc::mbar_init(&sm.v_full[s], 1);
      tc::mbar_init(&sm.v_empty[s], 1);
    }
    for (int i = 0; i < 2; i++) {
      tc::mbar_init(&sm.s_full[i], 1);
      tc::mbar_init(&sm.s_free[i], 8);   // one arrival per softmax warp
      tc::mbar_init(&sm.p_full[i], 8);
      tc::mbar_init(&sm.p_free[i], 1);
    }
    tc::fence_mbar_init();
    tc::prefetch_tmap(&tmap_q);
    tc::prefetch_tmap(&tmap_k);
    tc::prefetch_tmap(&tmap_v);
  }
  if (warp == 1) {
    tc::tmem_alloc(&sm.tmem_base, 512);   // S0 [0,128) S1 [128,256) O [256,384)
    tc::tmem_relinquish();
  }
  tc::tc_fence_before();
  __syncthreads();
  tc::tc_fence_after();
  const uint32_t tmem = sm.tmem_base;
  pdl_wait();   // Q and the chunk's K / V come from the previous kernel

  const int s = tile_seq[tile], q0 = tile_q0[tile];
  const int qlen = seq_qlen[s], qoff = seq_qoff[s], pos0 = seq_pos0[s];
  const int q_end = min(qlen, q0 + FA_QT);
  const int kmax = pos0 + q_end;                    // keys visible to the tile's last query
  const int NJ = (kmax + FA_KT - 1) / FA_KT;
  const int n_valid_pages = (kmax + FA_PG - 1) / FA_PG;
  const int* bt = block_table + (int64_t)s * bt_stride;

  if (warp == 0) {
    if (lane == 0) {
      tc::mbar_arrive_expect_tx(&sm.q_full, FA_QT * FA_D * 2);
      tc::tma_load_2d(sm.q[0], &tmap_q, &sm.q_full, h * FA_D, qoff + q0);
      tc::tma_load_2d(sm.q[1], &tmap_q, &sm.q_full, h * FA_D + 64, qoff + q0);
      for (int j = 0; j < NJ; j++) {
        // K of tile j: its single stage is free once S_{j-1} has been computed
        tc::mbar_wait(&sm.k_empty, (uint32_t)((j & 1) ^ 1), err);
        tc::mbar_arrive_expect_tx(&sm.k_full, FA_KT * FA_D * 2);
#pragma unroll 1
        for (int pi = 0; pi < FA_KT / FA_PG; pi++) {
          // pages past the visible keys repeat the last one (their keys are masked; the data stays finite)
          const int pidx = min(j * (FA_KT / FA_PG) + pi, n_valid_pages - 1);
          const int z = (layer * n_pages + bt[pidx]) * Hkv + g;
          for (int hd = 0; hd < 2; hd++) tma_load_3d(sm.k[hd] + pi * FA_PG * 64, &tmap_k, &sm.k_full, hd * 64, 0, z);
        }
        // V of tile j: stage j % 2, free once P.V_{j-2} has completed
        const int st = j % FA_STAGES;
        tc::mbar_wait(&sm.v_empty[st], (uint32_t)(((j / FA_STAGES) & 1) ^ 1), err);
        tc::mbar_arrive_expect_tx(&sm.v_full[st], FA_KT * FA_D * 2);
#pragma unroll 1
        for (int pi = 0; pi < FA_KT / FA_PG; pi++) {
          const int pidx = min(j * (FA_KT / FA_PG) + pi, n_valid_pages - 1);
          const int z = (layer * n_pages + bt[pidx]) * Hkv + g;
          for (int hd = 0; hd < 2; hd++) tma_load_3d(sm.v[st][hd] + pi * FA_PG * 64, &tmap_v, &sm.v_full[st], hd * 64, 0, z);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc_s = tc::idesc_bf16_f32(FA_QT, FA_KT);
      constexpr uint32_t idesc_pv = tc::idesc_bf16_f32(FA_QT, FA_D) | (1u << 16);   // B (V) MN-major
      const uint32_t to = tmem + 256u;
      tc::mbar_wait(&sm.q_full, 0, err);
      for (int j = 0; j <= NJ; j++) {
        if (j < NJ) {
          const int b = j & 1;
          tc::mbar_wait(&sm.k_full, (uint32_t)(j & 1), err);
          tc::mbar_wait(&sm.s_free[b], (uint32_t)(((j >> 1) & 1) ^ 1), err);
          tc::tc_fence_after();
          const uint32_t ts = tmem + (uint32_t)(b * 128);
#pragma unroll
          for (int hd = 0; hd < 2; hd++) {
            const uint64_t ad = tc::smem_desc_sw128(sm.q[hd]);
            const uint64_t bd = tc::smem_desc_sw128(sm.k[hd]);
#pragma unroll
            for (int kk = 0; kk < 4; kk++) tc::mma_bf16(ts, ad + 2 * kk, bd + 2 * kk, idesc_s, (hd | kk) != 0);
          }
          tc::mma_commit(&sm.s_full[b]);
          tc::mma_commit(&sm.k_empty);       // S_j done: K's stage takes tile j + 1
        }
        if (j > 0) {
          const int jj = j - 1, st = jj % FA_STAGES, pb = jj & 1;
          tc::mbar_wait(&sm.p_full[pb], (uint32_t)((jj >> 1) & 1), err);
          tc::mbar_wait(&sm.v_full[st], (uint32_t)((jj / FA_STAGES) & 1), err);
          tc::tc_fence_after();
#pragma unroll
          for (int ks = 0; ks < FA_KT / 16; ks++) {
            const uint64_t ad = tc::smem_desc_sw128(sm.p[pb][ks >> 2]) + 2 * (ks & 3);
            // 16 keys per step = 2 swizzle atoms of V; the two 64-column halves of the head dim are
            // 16 KB apart (LBO), 8-key groups 1 KB apart (SBO)
            const uint64_t bd = smem_desc_sw128_mn(sm.v[st][0] + ks * 16 * 64, FA_KT * 128, 1024);
            tc::mma_bf16(to, ad, bd, idesc_pv, (jj > 0 || ks != 0) ? 1u : 0u);
          }
          tc::mma_commit(&sm.p_free[pb]);    // P.V_jj done: O holds tiles <= jj, P buffer pb free
          tc::mma_commit(&sm.v_empty[st]);
        }
      }
    }
  } else {
    // softmax warps 2..9: TMEM lane quarter = warp % 4, key half kh = (warp - 2) / 4
    const int quarter = warp & 3, kh = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const int qi = q0 + r;
    const int pos = pos0 + qi;                       // keys [0, pos] are visible
    const int warp_pos = pos0 + q0 + quarter * 32;   // the smallest position among this warp's rows
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_off + 256u + (uint32_t)(kh * 64);   // this half's 64 columns of O
    float m = -INFINITY, l = 0.f;                    // exponent base (log2 units) and half-row sum against it
    for (int j = 0; j < NJ; j++) {
      const int b = j & 1;
      uint8_t* prow = reinterpret_cast<uint8_t*>(sm.p[b][kh]) + r * 128;
      tc::mbar_wait(&sm.s_full[b], (uint32_t)((j >> 1) & 1), err);
      tc::tc_fence_after();
      const uint32_t ts = tmem + lane_off + (uint32_t)(b * 128 + kh * 64);
      uint32_t sv[4][16];
#pragma unroll
      for (int c = 0; c < 4; c++) tc::tmem_ld16(ts + c * 16, sv[c]);
      tc::tmem_ld_wait();
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sm.s_free[b]);   // S is in registers: the buffer can take S_{j+2}
      const int k0 = j * FA_KT + kh * 64;
      // row max over four independent accumulators (a short dependency chain)
      float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
      const bool diag = k0 + 63 > warp_pos;   // warp-uniform
      if (diag) {   // a diagonal tile for this warp: mask keys past each row's position
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int e = 0; e < 16; e++) {
            const float x = k0 + c * 16 + e <= pos ? __uint_as_float(sv[c][e]) : -INFINITY;
            sv[c][e] = __float_as_uint(x);
            m4[e & 3] = fmaxf(m4[e & 3], x);
          }
      } else {
#pragma unroll
        for (int c = 0; c < 4; c++)
#pragma unroll
          for (int e = 0; e < 16; e++) m4[e & 3] = fmaxf(m4[e & 3], __uint_as_float(sv[c][e]));
      }
      float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
      // the other half's max of the same row (slots alternate by tile parity: a slot is rewritten
      // two tiles later, after a barrier the partner passes only once it has read it)
      sm.red[b][kh][r] = mx;
      asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
      mx = fmaxf(mx, sm.red[b][kh ^ 1][r]);
      const float m_new = fmaxf(m, mx * scale_log2);
      // move the base (and rescale O and l) only when some row of the warp outgrew the headroom;
      // the partner warp holds the same rows and values, so it takes the same decision
      const bool move = __any_sync(0xffffffffu, m_new > m + FA_HEADROOM);
      if (move) {
        const float f = ex2(m - m_new);   // 0 on the first tile
        if (j > 0) {
          // O must hold every earlier tile before it is rescaled: wait for P.V_{j-1}
          tc::mbar_wait(&sm.p_free[(j - 1) & 1], (uint32_t)(((j - 1) >> 1) & 1), err);
          tc::tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < 4; c++) {
            uint32_t ov[16];
            tc::tmem_ld16(tO + c * 16, ov);
            tc::tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 16; e++) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * f);
            tc::tmem_st16(tO + c * 16, ov);
          }
          tc::tmem_st_wait();
        }
        l *= f;
        m = m_new;
      }
      // this tile's P buffer is free once P.V_{j-2} has completed
      tc::mbar_wait(&sm.p_free[b], (uint32_t)(((j >> 1) & 1) ^ 1), err);
      float s4[4] = {0.f, 0.f, 0.f, 0.f};   // row sum, four independent accumulators
#pragma unroll
      for (int c = 0; c < 4; c++) {
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2) {
          const float p0 = ex2(fmaf(__uint_as_float(sv[c][e]), scale_log2, -m));
          const float p1 = ex2(fmaf(__uint_as_float(sv[c][e + 1]), scale_log2, -m));
          s4[(e >> 1) & 3] += p0 + p1;
          pk[e >> 1] = pack_bf16(p0, p1);
        }
        // keys kh*64 + c*16 .. +15: 16-byte chunks 2c and 2c+1 of the row in half kh, swizzled
        const int ch0 = 2 * c, ch1 = ch0 + 1;
        *reinterpret_cast<uint4*>(prow + 16 * (ch0 ^ (r & 7))) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
        *reinterpret_cast<uint4*>(prow + 16 * (ch1 ^ (r & 7))) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
      }
      l += (s4[0] + s4[1]) + (s4[2] + s4[3]);
      tc::tc_fence_before();
      tc::fence_proxy_async();   // generic-proxy stores of P -> visible to the tensor cores
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&sm.p_full[b]);
    }
    // the last P.V, then the row sum of both halves
    tc::mbar_wait(&sm.p_free[(NJ - 1) & 1], (uint32_t)(((NJ - 1) >> 1) & 1), err);
    tc::tc_fence_after();
    sm.lsum[kh][r] = l;
    asm volatile("bar.sync %0, 64;" ::"r"(1 + quarter) : "memory");
    l += sm.lsum[kh ^ 1][r];
    // every lane takes part in the warp-collective TMEM loads; rows past the chunk store nothing
    const bool store = qi < q_end;
    const float inv = l > 0.f ? 1.f / l : 0.f;
    __nv_bfloat16* dst = out + (int64_t)(qoff + (store ? qi : 0)) * ldo + (int64_t)h * FA_D + kh * 64;
#pragma unroll 1
    for (int c = 0; c < 4; c++) {
      uint32_t ov[16];
      tc::tmem_ld16(tO + c * 16, ov);
      tc::tmem_ld_wait();
      uint32_t w[8];
#pragma unroll
      for (int e = 0; e < 8; e++) w[e] = pack_bf16(__uint_as_float(ov[2 * e]) * inv, __uint_as_float(ov[2 * e + 1]) * inv);
      if (store) {
        *reinterpret_cast<uint4*>(dst + c * 16) = make_uint4(w[0], w[1], w[2], w[3]);
        *reinterpret_cast<uint4*>(dst + c * 16 + 8) = make_uint4(w[4], w[5], w[6], w[7]);
      }
    }
  }
  pdl_launch_dependents();
  tc::tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc::tc_fence_after();
    tc::tmem_dealloc(tmem, 512);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 fa_encode() {
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

}  // namespace

// q [T, Hq, D] bf16 (after RoPE); k_cache / v_cache: the whole cache [L, P, Hkv, 16, D] bf16; layer;
// block_table [S, W] int32; 128-query tiles (tile_seq, tile_q0, n_tiles) over the chunk's sequences
// (seq_qoff / seq_qlen / seq_pos0); out [T, Hq * D] bf16 (row stride ldo).
void prefill_attention_tc(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, int64_t layer,
                          torch::Tensor block_table, torch::Tensor tile_seq, torch::Tensor tile_q0, torch::Tensor seq_qoff,
                          torch::Tensor seq_qlen, torch::Tensor seq_pos0, int64_t n_tiles, torch::Tensor out,
                          c10::optional<torch::Tensor> err) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.is_contiguous() &&
                  q.size(2) == FA_D, "prefill_attention_tc: q [T, Hq, 128] bf16");
  TORCH_CHECK(k_cache.scalar_type() == torch::kBFloat16 && k_cache.dim() == 5 && k_cache.is_contiguous() &&
                  k_cache.size(3) == FA_PG && k_cache.size(4) == FA_D && v_cache.sizes() == k_cache.sizes() &&
                  v_cache.is_contiguous(), "prefill_attention_tc: caches [L, P, Hkv, 16, 128] bf16");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.stride(1) == 1 && out.stride(0) % 8 == 0,
              "prefill_attention_tc: out [T, >=Hq*128] bf16");
  const int T = (int)q.size(0), Hq = (int)q.size(1);
  const int L = (int)k_cache.size(0), P = (int)k_cache.size(1), Hkv = (int)k_cache.size(2);
  TORCH_CHECK(Hq % Hkv == 0 && layer >= 0 && layer < L, "prefill_attention_tc: heads / layer");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && block_table.stride(1) == 1, "prefill_attention_tc: bt");
  if (n_tiles <= 0 || T == 0) return;
  CUtensorMap mq, mk, mv;
  {
    cuuint64_t dims[2] = {(cuuint64_t)Hq * FA_D, (cuuint64_t)T};
    cuuint64_t strides[1] = {(cuuint64_t)Hq * FA_D * 2};
    cuuint32_t box[2] = {64, FA_QT};
    cuuint32_t estr[2] = {1, 1};
    CUresult rr = fa_encode()(&mq, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, q.data_ptr(), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(rr == CUDA_SUCCESS, "prefill_attention_tc: Q tensor map (", (int)rr, ")");
  }
  auto cache_map = [&](CUtensorMap& m, const torch::Tensor& t) {
    cuuint64_t dims[3] = {(cuuint64_t)FA_D, (cuuint64_t)FA_PG, (cuuint64_t)L * P * Hkv};
    cuuint64_t strides[2] = {(cuuint64_t)FA_D * 2, (cuuint64_t)FA_PG * FA_D * 2};
    cuuint32_t box[3] = {64, FA_PG, 1};
    cuuint32_t estr[3] = {1, 1, 1};
    CUresult rr = fa_encode()(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, t.data_ptr(), dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    TORCH_CHECK(rr == CUDA_SUCCESS, "prefill_attention_tc: KV tensor map (", (int)rr, ")");
  };
  cache_map(mk, k_cache);
  cache_map(mv, v_cache);
  const size_t smem = sizeof(FaSmem) + 1024;
  FAK_CUDA_CHECK(cudaFuncSetAttribute(k_prefill_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_tiles, (unsigned)Hq);
  cfg.blockDim = dim3(FA_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const float scale_log2 = (1.0f / sqrtf((float)FA_D)) * 1.4426950408889634f;
  int* ep = err.has_value() ? err->data_ptr<int>() : nullptr;
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_prefill_attn_tc, mq, mk, mv, (int)layer, P, Hkv, Hq,
                                    (const int*)block_table.data_ptr<int>(), (int)block_table.stride(0),
                                    (const int*)tile_seq.data_ptr<int>(), (const int*)tile_q0.data_ptr<int>(),
                                    (const int*)seq_qoff.data_ptr<int>(), (const int*)seq_qlen.data_ptr<int>(),
                                    (const int*)seq_pos0.data_ptr<int>(), reinterpret_cast<__nv_bfloat16*>(out.data_ptr<at::BFloat16>()),
                                    (int64_t)out.stride(0), scale_log2, ep));
}
