// In-kernel collectives over NVLink/NVSwitch peer memory for tensor-parallel decode.
//
// Every rank owns one symmetric buffer (same size and layout on all ranks, mapped into every
// peer's address space); kernels get the device array of the W peer base pointers.  Data moves
// with plain stores/loads to peer addresses; completion is signalled with flags in the same
// buffers:
//
//   flags region: uint32 [n_sites][MAX_CTAS][W]   (slot [site][cta][src] on the receiving rank)
//   a rank's CTA c publishes epoch e for site s by storing e (release, system scope) into
//   flags[s][c][me] of every peer, then waits (acquire, system scope) until its own
//   flags[s][c][r] >= e for every r.  Epochs come from a per-(site, cta) counter in local
//   memory, incremented by the kernel itself, so the kernels replay correctly inside CUDA graphs.
//
// Every wait is bounded: after a spin limit (a launch argument, default kSpinLimit polls) the kernel
// records error code 1 in `err` and continues, so a missing peer produces an error status on the
// host instead of a hung GPU; a short limit lets a test make the wait run out on purpose.
// No TMA or multicast loads are used here; peer memory is only touched by ordinary ld/st.
//
// Reference counterpart: the NCCL AllReduce/AllGather of internal/compute/cuda_nccl.cu:72-134 and
// the host-staged collective bridge internal/model/collective_bridge.go:103-120.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "common.cuh"

using namespace fak;

namespace {

constexpr int MAX_W = 8;
constexpr int MAX_CTAS = 128;
constexpr uint32_t kSpinLimit = 1u << 24;

FAK_DEV void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
FAK_DEV uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

struct Peers {
  uint8_t* base[MAX_W];  // symmetric buffer base of every rank
  uint32_t spin;         // polls of a flag before a wait gives up
};

// Cross-rank barrier for CTA `cta` at `site`: all threads of the CTA call it; prior writes of the
// CTA (to any rank) are visible to the peers once they pass it.
FAK_DEV void rank_barrier(const Peers& P, int64_t flags_off, int site, int cta, int me, int W, uint32_t* counters,
                          int* err) {
  __syncthreads();
  __shared__ uint32_t epoch_s;
  if (threadIdx.x == 0) {
    __threadfence_system();
    epoch_s = counters[site * MAX_CTAS + cta] + 1;
  }
  __syncthreads();
  const uint32_t epoch = epoch_s;
  const int64_t slot = ((int64_t)site * MAX_CTAS + cta) * MAX_W;
  if (threadIdx.x < W) {
    uint32_t* peer_flag = reinterpret_cast<uint32_t*>(P.base[threadIdx.x] + flags_off) + slot + me;
    st_release_sys(peer_flag, epoch);
  }
  if (threadIdx.x < W) {
    const uint32_t* mine = reinterpret_cast<const uint32_t*>(P.base[me] + flags_off) + slot + threadIdx.x;
    uint32_t i = 0;
    while (ld_acquire_sys(mine) < epoch) {
      if (++i > P.spin) {
        report_error(err, 1);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) counters[site * MAX_CTAS + cta] = epoch;
}

// ---- all-gather of per-rank column blocks of [B, row_bytes] byte matrices -------------------
// Up to two matrices (e.g. int8 codes and their (scale, sum) pairs) in one launch and one barrier.
// Rank `me` owns bytes [col0, col0 + ncols) of every row (in both the source and destination
// layout); it copies them from its local source into the same position of every rank's buffer.
struct AgSeg {
  const uint8_t* src;
  int64_t src_ld, dst_off, dst_ld, col0, ncols;
};

__global__ void k_p2p_allgather_cols(Peers P, AgSeg s0, AgSeg s1, int nseg, int B, int64_t flags_off, int site,
                                     int me, int W, uint32_t* counters, int* err) {
  pdl_wait();
  for (int k = 0; k < nseg; k++) {
    const AgSeg& g = k == 0 ? s0 : s1;
    const int64_t chunks = g.ncols >> 4;  // 16-byte chunks per row
    const int64_t total = (int64_t)B * chunks;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
      const int64_t b = i / chunks, c = i - b * chunks;
      const uint4 v = *reinterpret_cast<const uint4*>(g.src + b * g.src_ld + g.col0 + 16 * c);
      for (int r = 0; r < W; r++)
        *reinterpret_cast<uint4*>(P.base[r] + g.dst_off + b * g.dst_ld + g.col0 + 16 * c) = v;
    }
  }
  rank_barrier(P, flags_off, site, blockIdx.x, me, W, counters, err);
  pdl_launch_dependents();
}

// ---- one-shot all-reduce of fp32 partials, added into x ------------------------------------
// Every rank wrote its partial [n] into its own buffer at part_off; each element of x gets
// sum_r part_r (summed in rank order, so every rank computes bit-identical values).
__global__ void k_p2p_allreduce_add(Peers P, int64_t part_off, float* __restrict__ x, int64_t n, int64_t flags_off,
                                    int site, int me, int W, uint32_t* counters, int* err) {
  pdl_wait();
  rank_barrier(P, flags_off, site, blockIdx.x, me, W, counters, err);
  const int64_t n4 = n >> 2;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4; i += (int64_t)gridDim.x * blockDim.x) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < W; r++) {
      const float4 v = *reinterpret_cast<const float4*>(P.base[r] + part_off + 16 * i);
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    float4 xv = reinterpret_cast<float4*>(x)[i];
    xv.x += s.x; xv.y += s.y; xv.z += s.z; xv.w += s.w;
    reinterpret_cast<float4*>(x)[i] = xv;
  }
  pdl_launch_dependents();
}

// ---- prefill all-reduce: reduce + broadcast of owned tiles ----------------------------------
// The [M, N] fp32 output is cut into 128-row m-blocks and 256-column n-blocks; rank mb % W owns
// m-block mb.  Every rank has stored its partial of each tile into the owner's slot
// parts[src][owner-local row][N] and released the tile flag flags[mb][nb][src] with this call's
// epoch (the G_RS epilogue of gemm_tc.cu, or k_p2p_rs_push below).  For each owned tile, in the
// order the tiles are produced, a CTA waits (bounded) for the W flags, adds the partials in rank
// order to the residual x (a [M, N] fp32 array in every rank's peer buffer at x_off) and stores the
// sum into x on every rank; a cross-rank barrier per CTA then orders all broadcasts before the
// kernel ends, so every rank's x holds the full reduced rows.
constexpr int RS_BM = 128, RS_BN = 256;

FAK_DEV bool wait_flag_ge(const uint32_t* f, uint32_t v, uint32_t spin, int* err) {
  uint32_t i = 0;
  while (ld_acquire_sys(f) < v) {
    if (++i > spin) {
      report_error(err, 1);
      return false;
    }
  }
  return true;
}

// x_local != nullptr (sequence parallel): the residual is this rank's owned rows only, compacted
// ([MR, N], owner-local row index), updated in place with no broadcast and no closing barrier.
__global__ void __launch_bounds__(1024) k_p2p_rs_reduce(Peers P, int64_t parts_off, int64_t flags_off, int64_t x_off, int M, int N, int MR,
                                int me, int W, uint32_t epoch, int64_t bar_off, int site, uint32_t* counters,
                                int* err, float* __restrict__ x_local) {
  pdl_wait();
  const int n_m = (M + RS_BM - 1) / RS_BM, n_n = (N + RS_BN - 1) / RS_BN;
  const int own = me < n_m ? (n_m - 1 - me) / W + 1 : 0;   // owned m-blocks me, me + W, ...
  const uint8_t* mine = P.base[me];
  const float* parts = reinterpret_cast<const float*>(mine + parts_off);
  const float* xl = reinterpret_cast<const float*>(mine + x_off);
  for (int it = blockIdx.x; it < own * n_n; it += gridDim.x) {
    const int k = it % own, nb = it / own, mb = me + k * W;
    if (threadIdx.x < W)
      wait_flag_ge(reinterpret_cast<const uint32_t*>(mine + flags_off) + ((int64_t)mb * n_n + nb) * MAX_W + threadIdx.x,
                   epoch, P.spin, err);
    __syncthreads();
    const int rows = min(RS_BM, M - mb * RS_BM), cols4 = min(RS_BN, N - nb * RS_BN) >> 2;
    const int n4 = rows * cols4;
    // four float4 per thread in flight: the residual and every rank's partial of each are loaded
    // before any is added (same addition order per element)
    for (int e0 = threadIdx.x; e0 < n4; e0 += 4 * blockDim.x) {
      float4 acc[4];
      int64_t xi[4], pi[4];
#pragma unroll
      for (int u = 0; u < 4; u++) {
        const int e = min(e0 + u * (int)blockDim.x, n4 - 1);   // tail lanes repeat the last element
        const int rr = e / cols4, c = nb * RS_BN + 4 * (e - rr * cols4);
        xi[u] = x_local ? (int64_t)(k * RS_BM + rr) * N + c : (int64_t)(mb * RS_BM + rr) * N + c;
        pi[u] = (int64_t)(k * RS_BM + rr) * N + c;
        acc[u] = *reinterpret_cast<const float4*>((x_local ? x_local : xl) + xi[u]);
      }
      for (int r = 0; r < W; r++) {
        float4 v[4];
#pragma unroll
        for (int u = 0; u < 4; u++)
          v[u] = __ldcg(reinterpret_cast<const float4*>(parts + (int64_t)r * MR * N + pi[u]));
#pragma unroll
        for (int u = 0; u < 4; u++) {
          acc[u].x += v[u].x; acc[u].y += v[u].y; acc[u].z += v[u].z; acc[u].w += v[u].w;
        }
      }
#pragma unroll
      for (int u = 0; u < 4; u++) {
        if (e0 + u * (int)blockDim.x >= n4) break;
        if (x_local)
          *reinterpret_cast<float4*>(x_local + xi[u]) = acc[u];
        else
          for (int r = 0; r < W; r++)
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(P.base[r] + x_off) + xi[u]) = acc[u];
      }
    }
    __syncthreads();
  }
  if (!x_local) rank_barrier(P, bar_off, site, blockIdx.x, me, W, counters, err);
  pdl_launch_dependents();
}

// Sequence-parallel prefill: RMSNorm of this rank's owned rows (x_local [MR, N] compacted, `valid`
// of them real) into the bf16 shard of its peer buffer (shard_off, [MR, N]); once a 128-row block is
// written and fenced, its release flag (flags[m-block] = epoch) is stored into EVERY rank's buffer,
// so the next GEMM's producers (gemm_bf16_ag) wait on local memory.  One CTA per owned block, a
// warp per row.
__global__ void k_sp_rmsnorm_shard(Peers P, const float* __restrict__ x_local, const float* __restrict__ gamma,
                                   float eps, int N, int valid, int64_t shard_off, int64_t flags_off, int me, int W,
                                   uint32_t epoch) {
  pdl_wait();
  const int k = blockIdx.x, mb = me + k * W;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __nv_bfloat16* shard = reinterpret_cast<__nv_bfloat16*>(P.base[me] + shard_off);
  for (int rr = warp; rr < RS_BM; rr += nw) {
    const int lr = k * RS_BM + rr;
    if (lr >= valid) break;
    const float* xr = x_local + (int64_t)lr * N;
    float ss = 0.f;
    for (int c = lane * 4; c < N; c += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + c);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(ss / (float)N + eps);
    for (int c = lane * 4; c < N; c += 128) {
      const float4 v = *reinterpret_cast<const float4*>(xr + c);
      const float4 gm = *reinterpret_cast<const float4*>(gamma + c);
      __nv_bfloat162 a = __floats2bfloat162_rn(v.x * inv * gm.x, v.y * inv * gm.y);
      __nv_bfloat162 b = __floats2bfloat162_rn(v.z * inv * gm.z, v.w * inv * gm.w);
      uint2 pk;
      pk.x = *reinterpret_cast<uint32_t*>(&a);
      pk.y = *reinterpret_cast<uint32_t*>(&b);
      *reinterpret_cast<uint2*>(shard + (int64_t)lr * N + c) = pk;
    }
  }
  // the CTA barrier orders every thread's rows before the releasing threads' system fences
  __syncthreads();
  if (threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(reinterpret_cast<uint32_t*>(P.base[threadIdx.x] + flags_off) + mb, epoch);
  }
  pdl_launch_dependents();
}

// The reduce-scatter half for a partial that is not produced by a GEMM epilogue: part [M, N] fp32
// (local) is copied tile by tile into the owners' slots, each tile's flag released after its rows.
__global__ void k_p2p_rs_push(Peers P, const float* __restrict__ part, int M, int N, int MR, int64_t parts_off,
                              int64_t flags_off, int me, int W, uint32_t epoch) {
  pdl_wait();
  const int n_m = (M + RS_BM - 1) / RS_BM, n_n = (N + RS_BN - 1) / RS_BN;
  for (int t = blockIdx.x; t < n_m * n_n; t += gridDim.x) {
    const int mb = t % n_m, nb = t / n_m, owner = mb % W;
    float* dst = reinterpret_cast<float*>(P.base[owner] + parts_off);
    const int rows = min(RS_BM, M - mb * RS_BM), cols4 = min(RS_BN, N - nb * RS_BN) >> 2;
    for (int e = threadIdx.x; e < rows * cols4; e += blockDim.x) {
      const int rr = e / cols4, c = nb * RS_BN + 4 * (e - rr * cols4);
      const float4 v = *reinterpret_cast<const float4*>(part + (int64_t)(mb * RS_BM + rr) * N + c);
      *reinterpret_cast<float4*>(dst + ((int64_t)me * MR + (mb / W) * RS_BM + rr) * N + c) = v;
    }
    __syncthreads();   // every thread's rows of the tile, then one system fence and the flag
    if (threadIdx.x == 0) {
      __threadfence_system();
      st_release_sys(reinterpret_cast<uint32_t*>(P.base[owner] + flags_off) + ((int64_t)mb * n_n + nb) * MAX_W + me,
                     epoch);
    }
  }
  pdl_launch_dependents();
}

// ---- greedy sampling over vocab-sharded logits ---------------------------------------------
// Grid (rows, chunks).  Each CTA folds its chunk of the local vocabulary shard into one argmax key
// (global ids); the last CTA of a row (ticket) takes the row's key and exchanges it with the other
// ranks as one 16-byte line {key low, epoch, key high, epoch} stored into slot [parity][row][me]
// of every rank -- the epoch words travel in the same store as the key, so no fence or flag is
// needed -- then polls its own W slots (bounded) and every rank takes the same largest key.
// The epoch of a row counts launches in local memory (graph replays stay valid); slots alternate
// halves by epoch parity, so a rank one step ahead cannot overwrite a key a slower rank has not read.
constexpr int kArgmaxThreads = 256, kArgmaxPer = 4;   // a CTA's chunk: 256 x 4 float4 = 4096 floats

FAK_DEV void ll_store16(uint4* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
FAK_DEV uint4 ll_load16(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

template <bool VEC>
__global__ void k_p2p_argmax(Peers P, const float* __restrict__ logits, int64_t ld, int Vl, int64_t v_off,
                             int64_t cand_off, int* __restrict__ out, unsigned long long* __restrict__ keys,
                             int* __restrict__ tickets, uint32_t* __restrict__ epochs, int me, int W, int* err) {
  pdl_wait();
  const int b = blockIdx.x, chunk = kArgmaxThreads * kArgmaxPer * 4;
  const int i0 = blockIdx.y * chunk, i1 = min(Vl, i0 + chunk);
  const unsigned long long best =
      cta_best_key<VEC ? kArgmaxPer : 4 * kArgmaxPer, VEC>(logits + (int64_t)b * ld, i0, i1, (uint32_t)v_off);
  __shared__ int s_last;
  if (threadIdx.x == 0) {
    atomicMax(&keys[b], best);
    __threadfence();
    s_last = atomicAdd(&tickets[b], 1) == (int)gridDim.y - 1;
  }
  __syncthreads();
  pdl_launch_dependents();
  if (!s_last || threadIdx.x >= 32) return;
  const int lane = threadIdx.x;
  unsigned long long k = 0ull;
  uint32_t ep = 0;
  if (lane == 0) {
    __threadfence();
    k = atomicExch(&keys[b], 0ull);
    tickets[b] = 0;
    ep = epochs[b] + 1;
  }
  k = __shfl_sync(0xffffffffu, k, 0);
  ep = __shfl_sync(0xffffffffu, ep, 0);
  const int64_t half = (int64_t)(ep & 1u) * MAX_CTAS * MAX_W;
  if (lane < W) {   // lane r pushes to rank r, then reads rank r's key from its own buffer
    const uint4 line = make_uint4((uint32_t)(k & 0xFFFFFFFFull), ep, (uint32_t)(k >> 32), ep);
    ll_store16(reinterpret_cast<uint4*>(P.base[lane] + cand_off) + half + (int64_t)b * MAX_W + me, line);
  }
  unsigned long long kr = 0ull;
  if (lane < W) {
    const uint4* src = reinterpret_cast<const uint4*>(P.base[me] + cand_off) + half + (int64_t)b * MAX_W + lane;
    uint4 v;
    uint32_t it = 0;
    while (true) {
      v = ll_load16(src);
      if (v.y == ep && v.w == ep) break;
      if (++it > P.spin) {
        report_error(err, 1);
        break;
      }
    }
    kr = ((unsigned long long)v.z << 32) | v.x;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long t = __shfl_xor_sync(0xffffffffu, kr, o);
    kr = t > kr ? t : kr;
  }
  if (lane == 0) {
    out[b] = argmax_key_index(kr);
    epochs[b] = ep;
  }
}

// ---- MoE combine fused with the expert-parallel all-reduce -----------------------------------
// Expert parallelism with the residual stream replicated on every rank (attention is head-parallel),
// so a token's activation is already on every rank and the grouped expert GEMV gathers the rows it
// needs locally: the only cross-rank step is the combine.  CTA c owns elements [c * chunk, ...) of
// the flattened [B, d] output: it sums, for each element, the router-weighted outputs of the experts
// in this rank's band (the token's k slots in order), pushes those partials into slot [me] of every
// rank's buffer (half `parity` of [2][W][B*d]), crosses the per-(site, CTA) barrier, and adds the
// rank-order sum of the W slots to the residual -- bit-identical on every rank.  Consecutive MoE
// layers alternate halves, so a fast rank's next layer cannot overwrite partials a slow rank has
// not summed: reaching the next use of a half requires passing the layer in between.
__global__ void k_moe_combine_ar(Peers P, const float* __restrict__ out, const int* __restrict__ ids,
                                 const float* __restrict__ wts, int k, int e0, int E_local, float* __restrict__ x,
                                 int B, int d, int64_t parts_off, int parity, int64_t flags_off, int site, int me, int W,
                                 uint32_t* counters, int* err) {
  pdl_wait();
  const int64_t n = (int64_t)B * d;
  const int64_t chunk = (n + gridDim.x - 1) / gridDim.x;
  const int64_t i0 = blockIdx.x * chunk, i1 = min(n, i0 + chunk);
  const int64_t half = (int64_t)parity * W * n;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    const int b = (int)(i / d), c = (int)(i - (int64_t)b * d);
    float s = 0.f;
    for (int j = 0; j < k; j++) {
      const int e = ids[b * k + j] - e0;
      if (e >= 0 && e < E_local) s += wts[b * k + j] * out[((int64_t)b * k + j) * d + c];
    }
    for (int r = 0; r < W; r++) reinterpret_cast<float*>(P.base[r] + parts_off)[half + (int64_t)me * n + i] = s;
  }
  rank_barrier(P, flags_off, site, blockIdx.x, me, W, counters, err);
  const float* mine = reinterpret_cast<const float*>(P.base[me] + parts_off) + half;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < W; r++) s += __ldcg(mine + (int64_t)r * n + i);
    x[i] += s;
  }
  pdl_launch_dependents();
}

Peers make_peers(torch::Tensor ptrs, int64_t spin_limit) {
  TORCH_CHECK(ptrs.scalar_type() == torch::kInt64 && ptrs.numel() <= MAX_W, "peer pointer table");
  TORCH_CHECK(spin_limit >= 0 && spin_limit <= 0xffffffffll, "spin limit");
  auto h = ptrs.cpu();
  Peers P{};
  P.spin = spin_limit > 0 ? (uint32_t)spin_limit : kSpinLimit;
  for (int i = 0; i < ptrs.numel(); i++) P.base[i] = reinterpret_cast<uint8_t*>(h.data_ptr<int64_t>()[i]);
  return P;
}

cudaLaunchConfig_t pdl_cfg(dim3 grid, dim3 block, cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

}  // namespace

// peers: int64 [W] host tensor of symmetric buffer bases; counters: int32 [n_sites*64] local
// device tensor (zero-initialised once); err: int32 [1] device.
// Segments: one or two (src, src_ld, dst_off, dst_ld, col0, ncols) column blocks gathered in one launch.
void p2p_allgather_cols(torch::Tensor peers, torch::Tensor src, int64_t src_ld, int64_t dst_off, int64_t dst_ld,
                        int64_t col0, int64_t ncols, int64_t B, int64_t flags_off, int64_t site, int64_t me,
                        torch::Tensor counters, torch::Tensor err, int64_t ctas, c10::optional<torch::Tensor> src2,
                        int64_t src2_ld, int64_t dst2_off, int64_t dst2_ld, int64_t col2, int64_t ncols2,
                        int64_t spin_limit) {
  const int W = (int)peers.numel();
  auto check = [](int64_t n, int64_t c, int64_t sl, int64_t dl, int64_t off) {
    TORCH_CHECK(n % 16 == 0 && c % 16 == 0 && sl % 16 == 0 && dl % 16 == 0 && off % 16 == 0,
                "allgather: 16-byte granularity");
  };
  check(ncols, col0, src_ld, dst_ld, dst_off);
  TORCH_CHECK(ctas >= 1 && ctas <= MAX_CTAS, "allgather: 1..128 CTAs");
  AgSeg s0{(const uint8_t*)src.data_ptr(), src_ld, dst_off, dst_ld, col0, ncols};
  AgSeg s1 = s0;
  int nseg = 1;
  if (src2.has_value()) {
    check(ncols2, col2, src2_ld, dst2_ld, dst2_off);
    s1 = AgSeg{(const uint8_t*)src2->data_ptr(), src2_ld, dst2_off, dst2_ld, col2, ncols2};
    nseg = 2;
  }
  Peers P = make_peers(peers, spin_limit);
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_cfg(dim3((unsigned)ctas), dim3(256), attr);
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_p2p_allgather_cols, P, s0, s1, nseg, (int)B, flags_off, (int)site,
                                    (int)me, W, (uint32_t*)counters.data_ptr<int>(), err.data_ptr<int>()));
}

void p2p_allreduce_add(torch::Tensor peers, int64_t part_off, torch::Tensor x, int64_t n, int64_t flags_off,
                       int64_t site, int64_t me, torch::Tensor counters, torch::Tensor err, int64_t ctas,
                       int64_t spin_limit) {
  const int W = (int)peers.numel();
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.numel() >= n && n % 4 == 0, "x");
  TORCH_CHECK(part_off % 16 == 0, "partials must be 16-byte aligned");
  TORCH_CHECK(ctas >= 1 && ctas <= MAX_CTAS, "allreduce: 1..128 CTAs");
  Peers P = make_peers(peers, spin_limit);
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_cfg(dim3((unsigned)ctas), dim3(256), attr);
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_p2p_allreduce_add, P, part_off, x.data_ptr<float>(), n, flags_off,
                                    (int)site, (int)me, W, (uint32_t*)counters.data_ptr<int>(), err.data_ptr<int>()));
}

// Completes the prefill all-reduce started by gemm_bf16_rs / p2p_rs_push: x (at x_off in every
// rank's peer buffer, [M, N] fp32) += sum over ranks of the partials; site: barrier site for the end.
void p2p_rs_reduce(torch::Tensor peers, int64_t parts_off, int64_t flags_off, int64_t x_off, int64_t M, int64_t N,
                   int64_t MR, int64_t me, int64_t epoch, int64_t bar_off, int64_t site, torch::Tensor counters,
                   torch::Tensor err, int64_t ctas, int64_t spin_limit, c10::optional<torch::Tensor> x_local) {
  const int W = (int)peers.numel();
  TORCH_CHECK(N % 4 == 0 && parts_off % 16 == 0 && x_off % 16 == 0 && flags_off % 4 == 0, "rs_reduce: alignment");
  TORCH_CHECK(ctas >= 1 && ctas <= MAX_CTAS, "rs_reduce: 1..128 CTAs");
  TORCH_CHECK(MR >= ((M + RS_BM - 1) / RS_BM + W - 1) / W * RS_BM, "rs_reduce: MR");
  if (M == 0) return;
  Peers P = make_peers(peers, spin_limit);
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_cfg(dim3((unsigned)ctas), dim3(1024), attr);
  float* xl = nullptr;
  if (x_local.has_value()) {
    TORCH_CHECK(x_local->is_cuda() && x_local->scalar_type() == torch::kFloat32 && x_local->is_contiguous() &&
                    x_local->numel() >= MR * N, "rs_reduce: x_local [MR, N] f32");
    xl = x_local->data_ptr<float>();
  }
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_p2p_rs_reduce, P, parts_off, flags_off, x_off, (int)M, (int)N, (int)MR,
                                    (int)me, W, (uint32_t)epoch, bar_off, (int)site,
                                    (uint32_t*)counters.data_ptr<int>(), err.data_ptr<int>(), xl));
}

void sp_rmsnorm_shard(torch::Tensor peers, torch::Tensor x_local, torch::Tensor gamma, double eps, int64_t valid,
                      int64_t shard_off, int64_t flags_off, int64_t me, int64_t epoch) {
  const int W = (int)peers.numel();
  TORCH_CHECK(x_local.is_cuda() && x_local.scalar_type() == torch::kFloat32 && x_local.dim() == 2 &&
                  x_local.is_contiguous() && x_local.size(1) % 128 == 0, "sp_rmsnorm: x_local [MR, N] f32, N % 128");
  TORCH_CHECK(gamma.scalar_type() == torch::kFloat32 && gamma.numel() >= x_local.size(1), "sp_rmsnorm: gamma");
  TORCH_CHECK(shard_off % 16 == 0 && valid <= x_local.size(0), "sp_rmsnorm: shard / rows");
  const int blocks = (int)((valid + RS_BM - 1) / RS_BM);
  if (blocks == 0) return;
  Peers P = make_peers(peers, 0);
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_cfg(dim3((unsigned)blocks), dim3(512), attr);
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_sp_rmsnorm_shard, P, (const float*)x_local.data_ptr<float>(),
                                    (const float*)gamma.data_ptr<float>(), (float)eps, (int)x_local.size(1),
                                    (int)valid, shard_off, flags_off, (int)me, W, (uint32_t)epoch));
}

void p2p_rs_push(torch::Tensor peers, torch::Tensor part, int64_t MR, int64_t parts_off, int64_t flags_off, int64_t me,
                 int64_t epoch) {
  const int W = (int)peers.numel();
  TORCH_CHECK(part.is_cuda() && part.scalar_type() == torch::kFloat32 && part.dim() == 2 && part.is_contiguous() &&
                  part.size(1) % 4 == 0, "rs_push: part [M, N] f32 contiguous, N % 4 == 0");
  const int M = (int)part.size(0), N = (int)part.size(1);
  TORCH_CHECK(MR >= ((M + RS_BM - 1) / RS_BM + W - 1) / W * RS_BM && parts_off % 16 == 0, "rs_push: MR / offset");
  if (M == 0) return;
  Peers P = make_peers(peers, 0);
  const int tiles = ((M + RS_BM - 1) / RS_BM) * ((N + RS_BN - 1) / RS_BN);
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_cfg(dim3((unsigned)std::min(tiles, 148)), dim3(256), attr);
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_p2p_rs_push, P, (const float*)part.data_ptr<float>(), M, N, (int)MR,
                                    parts_off, flags_off, (int)me, W, (uint32_t)epoch));
}

// logits [B, >= Vl] f32 (this rank's vocabulary shard, global ids v_off + i); cand_off: the
// [2][MAX_CTAS][MAX_W] 16-byte line slots of the peer buffers; keys / tickets: local [B] scratch left
// at zero; epochs: local [MAX_CTAS] launch counters.
void p2p_argmax(torch::Tensor peers, torch::Tensor logits, int64_t Vl, int64_t v_off, int64_t cand_off,
                torch::Tensor out, int64_t B, torch::Tensor keys, torch::Tensor tickets, torch::Tensor epochs,
                int64_t me, torch::Tensor err, int64_t spin_limit) {
  const int W = (int)peers.numel();
  TORCH_CHECK(logits.scalar_type() == torch::kFloat32 && logits.stride(1) == 1, "logits");
  TORCH_CHECK(B >= 1 && B <= MAX_CTAS, "argmax: batch 1..128");
  TORCH_CHECK(cand_off % 16 == 0, "argmax: candidate slots 16-byte aligned");
  TORCH_CHECK(keys.scalar_type() == torch::kInt64 && keys.numel() >= B && tickets.scalar_type() == torch::kInt32 &&
                  tickets.numel() >= B, "argmax: keys [B] int64, tickets [B] int32");
  TORCH_CHECK(epochs.scalar_type() == torch::kInt32 && epochs.numel() >= MAX_CTAS, "argmax: epochs [128] int32");
  TORCH_CHECK(v_off >= 0 && v_off + Vl < 0xFFFFFFFFll, "argmax: ids fit 32 bits");
  Peers P = make_peers(peers, spin_limit);
  const int chunk = kArgmaxThreads * kArgmaxPer * 4;
  const bool vec = logits.stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(logits.data_ptr()) % 16 == 0;
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_cfg(dim3((unsigned)B, (unsigned)((Vl + chunk - 1) / chunk)), dim3(kArgmaxThreads), attr);
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, vec ? k_p2p_argmax<true> : k_p2p_argmax<false>, P,
                                    (const float*)logits.data_ptr<float>(), (int64_t)logits.stride(0), (int)Vl, v_off,
                                    cand_off, out.data_ptr<int>(),
                                    reinterpret_cast<unsigned long long*>(keys.data_ptr<int64_t>()),
                                    tickets.data_ptr<int>(), reinterpret_cast<uint32_t*>(epochs.data_ptr<int>()),
                                    (int)me, W, err.data_ptr<int>()));
}

// out [B*k, d] f32 (expert outputs per (token, slot)); ids / wts [B, k]; x [B, d] f32 (residual, updated);
// parts_off: [2][W][B*d] f32 region of the peer buffers; site: this layer's barrier site.
void p2p_moe_combine_ar(torch::Tensor peers, torch::Tensor out, torch::Tensor ids, torch::Tensor wts, int64_t k,
                        int64_t e0, int64_t E_local, torch::Tensor x, int64_t B, int64_t parts_off, int64_t parity,
                        int64_t flags_off, int64_t site, int64_t me, torch::Tensor counters, torch::Tensor err,
                        int64_t ctas, int64_t spin_limit) {
  const int W = (int)peers.numel();
  TORCH_CHECK(out.scalar_type() == torch::kFloat32 && out.is_contiguous() && out.size(0) >= B * k, "moe_combine_ar: out");
  TORCH_CHECK(x.scalar_type() == torch::kFloat32 && x.is_contiguous() && x.size(0) >= B, "moe_combine_ar: x");
  TORCH_CHECK(ids.scalar_type() == torch::kInt32 && wts.scalar_type() == torch::kFloat32, "moe_combine_ar: ids / wts");
  TORCH_CHECK(parts_off % 16 == 0 && (parity == 0 || parity == 1), "moe_combine_ar: parts layout");
  TORCH_CHECK(ctas >= 1 && ctas <= MAX_CTAS, "moe_combine_ar: 1..128 CTAs");
  if (B <= 0) return;
  Peers P = make_peers(peers, spin_limit);
  cudaLaunchAttribute attr[1];
  auto cfg = pdl_cfg(dim3((unsigned)ctas), dim3(256), attr);
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_moe_combine_ar, P, (const float*)out.data_ptr<float>(),
                                    (const int*)ids.data_ptr<int>(), (const float*)wts.data_ptr<float>(), (int)k,
                                    (int)e0, (int)E_local, x.data_ptr<float>(), (int)B, (int)x.size(1), parts_off,
                                    (int)parity, flags_off, (int)site, (int)me, W, (uint32_t*)counters.data_ptr<int>(),
                                    err.data_ptr<int>()));
}
