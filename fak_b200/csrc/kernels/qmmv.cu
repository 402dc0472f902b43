// Quantized matrix x (few tokens) product on the integer tensor cores, for decode batches.
//
// y[b, n] = sum_k W[n, k] x[b, k], W in GGML Q4_K / Q6_K / Q8_0 blocks (16-byte row pitch),
// x pre-quantized to int8 per 32-element block with (scale, sum of the dequantized block), B <= 8.
//
// Each CTA owns one 16-row tile; its 8 warps split K.  Per quantization sub-block the weights
// of the 16 rows form the A operand of an integer MMA (m16n8k32 for 32-element sub-blocks,
// m16n8k16 for Q6_K's 16-element ones) and the 8 token columns the B operand, so one
// instruction does 16 x 8 x 32 multiply-adds; the int32 fragment is then scaled by
// (weight block scale x activation block scale) and accumulated in fp32:
//   Q4_K:  d*sc * dx * sum(q*qx)  -  dmin*m * dx * sum(qx)  (q in 0..15)
//   Q6_K:  d*sc * dx * sum((q-32)*qx)
//   Q8_0:  dw * dx * sum(qw*qx)
// The k order inside a sub-block is free (it is summed), so each thread loads 8 contiguous
// weight bytes and the matching 8 contiguous activation bytes instead of the ISA's k pattern.
// This replaces the CUDA-core dp4a inner product, whose integer op count per weight grows
// with the batch; here it is flat in B.  Partial sums of the 8 warps meet in shared memory.
// Epilogue: bias, residual add (in place), or SwiGLU over 8-row interleaved gate/up blocks.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "tc.cuh"

using namespace fak;

namespace {

enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2 };
constexpr int WARPS = 8;

FAK_DEV void mma_s8_16832(int (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
FAK_DEV void mma_s8_16816(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
  asm volatile("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%0,%1,%2,%3};"
               : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
               : "r"(a0), "r"(a1), "r"(b0));
}

// Q4_K: unpack the eight 6-bit (scale, min) pairs of a super-block from its 12 packed bytes
// (words s0 = bytes 0-3, s1 = 4-7, s2 = 8-11) four at a time: byte j of sc_lo/m_lo holds the
// pair of sub-block j, byte j of sc_hi/m_hi the pair of sub-block 4+j.
FAK_DEV void q4k_unpack_scales(uint32_t s0, uint32_t s1, uint32_t s2, uint32_t& sc_lo, uint32_t& sc_hi,
                               uint32_t& m_lo, uint32_t& m_hi) {
  sc_lo = s0 & 0x3F3F3F3Fu;
  m_lo = s1 & 0x3F3F3F3Fu;
  sc_hi = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
  m_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
}
FAK_DEV float byte_f(uint32_t w, int i) { return i2f_exact22((int)((w >> (8 * i)) & 0xffu)); }

// Bytes per quantization "super" unit that one warp consumes per stage (256 weights for the
// K-quants, 8 Q8_0 blocks = 256 weights), and super units per pipeline stage (one per warp).
template <int QT>
struct QInfo;
template <> struct QInfo<QT_Q4_K> { static constexpr int BYTES = 144; };
template <> struct QInfo<QT_Q6_K> { static constexpr int BYTES = 210; };
template <> struct QInfo<QT_Q8_0> { static constexpr int BYTES = 8 * 34; };

FAK_DEV uint32_t lds_u32_a2(const uint8_t* p) {  // 4 bytes at a 2-byte-aligned shared address
  uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if ((a & 3) == 0) return *reinterpret_cast<const uint32_t*>(p);
  const uint16_t* h = reinterpret_cast<const uint16_t*>(p);
  return (uint32_t)h[0] | ((uint32_t)h[1] << 16);
}
FAK_DEV uint2 lds_u64_a2(const uint8_t* p) { return make_uint2(lds_u32_a2(p), lds_u32_a2(p + 4)); }


// One super unit (256 weights) of the 16-row tile, rows g and g+8, everything from shared memory.
// xs: token g's activations at this unit; dsu: (scale, sum) row base at this unit's first block.
template <int QT>
FAK_DEV void tile_unit(const uint8_t* ua, const uint8_t* ub, const int8_t* xs, const float2* d0, const float2* d1,
                       int nvalid_blk, bool tok_ok, int t, float (&acc)[4]) {
  auto xload8 = [&](int off) -> uint2 {
    return tok_ok ? *reinterpret_cast<const uint2*>(xs + off) : make_uint2(0u, 0u);
  };
  if constexpr (QT == QT_Q4_K) {
    const uint4 ha = *reinterpret_cast<const uint4*>(ua), hb = *reinterpret_cast<const uint4*>(ub);
    const float da = __half2float(__ushort_as_half((uint16_t)(ha.x & 0xffff)));
    const float dma = __half2float(__ushort_as_half((uint16_t)(ha.x >> 16)));
    const float db = __half2float(__ushort_as_half((uint16_t)(hb.x & 0xffff)));
    const float dmb = __half2float(__ushort_as_half((uint16_t)(hb.x >> 16)));
    uint32_t sca_lo, sca_hi, ma_lo, ma_hi, scb_lo, scb_hi, mb_lo, mb_hi;
    q4k_unpack_scales(ha.y, ha.z, ha.w, sca_lo, sca_hi, ma_lo, ma_hi);
    q4k_unpack_scales(hb.y, hb.z, hb.w, scb_lo, scb_hi, mb_lo, mb_hi);
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const uint2 qa = *reinterpret_cast<const uint2*>(ua + 16 + 32 * c + 8 * t);
      const uint2 qb = *reinterpret_cast<const uint2*>(ub + 16 + 32 * c + 8 * t);
#pragma unroll
      for (int hi = 0; hi < 2; hi++) {
        const int j = 2 * c + hi;
        const uint2 xb = xload8(32 * j + 8 * t);
        const int sh = 4 * hi;
        uint32_t a[4] = {(qa.x >> sh) & 0x0F0F0F0Fu, (qb.x >> sh) & 0x0F0F0F0Fu, (qa.y >> sh) & 0x0F0F0F0Fu,
                         (qb.y >> sh) & 0x0F0F0F0Fu};
        int cc[4] = {0, 0, 0, 0};
        mma_s8_16832(cc, a, xb.x, xb.y);
        const float2 x0 = d0[j], x1 = d1[j];
        const float fa = da * byte_f(j < 4 ? sca_lo : sca_hi, j & 3), fb = db * byte_f(j < 4 ? scb_lo : scb_hi, j & 3);
        const float ma_ = dma * byte_f(j < 4 ? ma_lo : ma_hi, j & 3), mb_ = dmb * byte_f(j < 4 ? mb_lo : mb_hi, j & 3);
        acc[0] = fmaf(fa * x0.x, i2f_exact22(cc[0]), fmaf(-ma_, x0.y, acc[0]));
        acc[1] = fmaf(fa * x1.x, i2f_exact22(cc[1]), fmaf(-ma_, x1.y, acc[1]));
        acc[2] = fmaf(fb * x0.x, i2f_exact22(cc[2]), fmaf(-mb_, x0.y, acc[2]));
        acc[3] = fmaf(fb * x1.x, i2f_exact22(cc[3]), fmaf(-mb_, x1.y, acc[3]));
      }
    }
  } else if constexpr (QT == QT_Q8_0) {
#pragma unroll
    for (int bi = 0; bi < 8; bi++) {
      if (bi >= nvalid_blk) break;
      const uint8_t* pa = ua + 34 * bi;
      const uint8_t* pb = ub + 34 * bi;
      const uint2 qa = lds_u64_a2(pa + 2 + 8 * t), qb = lds_u64_a2(pb + 2 + 8 * t);
      const float da = half_bits_to_float(*reinterpret_cast<const uint16_t*>(pa));
      const float db = half_bits_to_float(*reinterpret_cast<const uint16_t*>(pb));
      const uint2 xb = xload8(32 * bi + 8 * t);
      uint32_t a[4] = {qa.x, qb.x, qa.y, qb.y};
      int cc[4] = {0, 0, 0, 0};
      mma_s8_16832(cc, a, xb.x, xb.y);
      const float2 x0 = d0[bi], x1 = d1[bi];
      acc[0] = fmaf(da * x0.x, i2f_exact22(cc[0]), acc[0]);
      acc[1] = fmaf(da * x1.x, i2f_exact22(cc[1]), acc[1]);
      acc[2] = fmaf(db * x0.x, i2f_exact22(cc[2]), acc[2]);
      acc[3] = fmaf(db * x1.x, i2f_exact22(cc[3]), acc[3]);
    }
  } else {  // Q6_K
    const float da = half_bits_to_float(*reinterpret_cast<const uint16_t*>(ua + 208));
    const float db = half_bits_to_float(*reinterpret_cast<const uint16_t*>(ub + 208));
#pragma unroll
    for (int n = 0; n < 2; n++) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int l0 = 16 * h + 4 * t;
        const uint32_t la0 = lds_u32_a2(ua + n * 64 + l0), la1 = lds_u32_a2(ua + n * 64 + 32 + l0);
        const uint32_t lb0 = lds_u32_a2(ub + n * 64 + l0), lb1 = lds_u32_a2(ub + n * 64 + 32 + l0);
        const uint32_t hha = lds_u32_a2(ua + 128 + n * 32 + l0), hhb = lds_u32_a2(ub + 128 + n * 32 + l0);
#pragma unroll
        for (int k = 0; k < 4; k++) {
          const uint32_t la = (k & 1) ? la1 : la0, lb = (k & 1) ? lb1 : lb0;
          const int ls = (k >> 1) * 4, hs = 2 * k;
          uint32_t qa4 = ((la >> ls) & 0x0F0F0F0Fu) | (((hha >> hs) & 0x03030303u) << 4);
          uint32_t qb4 = ((lb >> ls) & 0x0F0F0F0Fu) | (((hhb >> hs) & 0x03030303u) << 4);
          qa4 = __vsub4(qa4, 0x20202020u);
          qb4 = __vsub4(qb4, 0x20202020u);
          const int e0 = n * 128 + 32 * k + 16 * h;
          const uint32_t xb = tok_ok ? *reinterpret_cast<const uint32_t*>(xs + e0 + 4 * t) : 0u;
          int cc[4] = {0, 0, 0, 0};
          mma_s8_16816(cc, qa4, qb4, xb);
          const int sub = e0 >> 4;
          const float sa = da * i2f_exact22((int)(int8_t)ua[192 + sub]);
          const float sbv = db * i2f_exact22((int)(int8_t)ub[192 + sub]);
          const float2 x0 = d0[e0 >> 5], x1 = d1[e0 >> 5];
          acc[0] = fmaf(sa * x0.x, i2f_exact22(cc[0]), acc[0]);
          acc[1] = fmaf(sa * x1.x, i2f_exact22(cc[1]), acc[1]);
          acc[2] = fmaf(sbv * x0.x, i2f_exact22(cc[2]), acc[2]);
          acc[3] = fmaf(sbv * x1.x, i2f_exact22(cc[3]), acc[3]);
        }
      }
    }
  }
}

// 1-D TMA bulk copy global -> shared, completing `bytes` transaction bytes on an mbarrier
// (both addresses 16-byte aligned, size a multiple of 16; no cluster multicast).
FAK_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          tc::smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(tc::smem_addr(bar))
      : "memory");
}

// Persistent kernel: CTA c walks the 16-row tiles c, c + gridDim.x, ...  A work item is one
// tile x one K range.  When the 16 rows fit in one ring slot the item is the whole tile and moves
// as ONE contiguous 1-D TMA bulk copy (rows are contiguous at the device row pitch, which is
// 16 mod 128 bytes so consecutive rows land on different banks); otherwise the K range is cut into
// chunks and each row's chunk is one bulk copy.  Activations and their (scale, sum) pairs for the
// item's K range ride along; when every item spans all of K they are copied only for the first
// ring round and stay resident.  One thread issues all copies (completion on the slot's mbarrier)
// and keeps STAGES-1 items in flight across tile boundaries.  Warp w consumes super units
// w, w+8, ... of each item; a __syncthreads per item retires the slot and, at a tile's last item,
// publishes the per-warp partial sums that warp 0 reduces for the epilogue.
struct ItemGeom {
  int units;        // super units per item
  int items;        // items per tile
  int wrow;         // shared-memory row stride of the weight slot
  int wbytes;       // weight bytes per slot
  int xbytes;       // activation bytes per token per item
  bool whole;       // item = whole tile (one contiguous copy)
};

template <int QT, int STAGES>
__global__ void __launch_bounds__(WARPS * 32)
k_qmmv(const uint8_t* __restrict__ W, int N, int K, int64_t pitch, const int8_t* __restrict__ qx,
       const float2* __restrict__ ds, int B, float* __restrict__ y, int64_t ldy, const float* __restrict__ bias,
       int epi, int* __restrict__ err, int flags, ItemGeom geo) {
  constexpr int UB = QInfo<QT>::BYTES;   // bytes per super unit
  extern __shared__ __align__(128) uint8_t sm[];
  __shared__ float red[2][WARPS][32][4];
  __shared__ uint64_t full[STAGES];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int64_t nblk = K >> 5;
  const int n_units = (K + 255) >> 8;               // 256-weight super units per row (Q8_0: last may be partial)
  const int64_t row_bytes = QT == QT_Q8_0 ? nblk * 34 : (int64_t)n_units * UB;
  const int xs_stride = geo.xbytes + 32;            // token rows of the activation slot (32 mod 128 B apart)
  const int slot_bytes = geo.wbytes + B * (xs_stride + geo.xbytes / 4);
  const int n_tiles = (N + 15) >> 4;
  const int my_tiles = n_tiles > (int)blockIdx.x ? (n_tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  const int n_items = my_tiles * geo.items;
  if (threadIdx.x == 0) {
    for (int i = 0; i < STAGES; i++) tc::mbar_init(&full[i], 1);
    tc::fence_mbar_init();
  }
  __syncthreads();

  auto item_tile = [&](int it) { return (int)blockIdx.x + (it / geo.items) * (int)gridDim.x; };
  auto acts_needed = [&](int it) { return geo.items > 1 || it < STAGES; };
  auto act_bytes = [&](int it) -> uint32_t {
    const int64_t k0 = (int64_t)(it % geo.items) * geo.units * 256;
    return (uint32_t)min((int64_t)geo.xbytes, (int64_t)K - k0);  // multiple of 64
  };
  auto issue_weights = [&](int it) {
    if (it >= n_items) return;
    const int part = it % geo.items, r0 = item_tile(it) * 16;
    uint8_t* dst = sm + (size_t)(it % STAGES) * slot_bytes;
    uint32_t wtx;
    if (geo.whole) {
      // rows r0..r0+15 back to back (only the rows that exist for the tail tile; the MMA rows past
      // N then read stale slot bytes, which only feed outputs that are never stored)
      wtx = (uint32_t)(min(16, N - r0) * pitch);
    } else {
      const int64_t off = (int64_t)part * geo.units * UB;
      wtx = 16u * (uint32_t)((min((int64_t)geo.units * UB, row_bytes - off) + 15) & ~int64_t(15));
    }
    const uint32_t xb = acts_needed(it) ? act_bytes(it) : 0u;
    tc::mbar_arrive_expect_tx(&full[it % STAGES], wtx + B * (xb + xb / 4));
    if (geo.whole) {
      bulk_g2s(dst, W + (int64_t)r0 * pitch, wtx, &full[it % STAGES]);
    } else {
      const int64_t off = (int64_t)part * geo.units * UB;
      const uint32_t wb = wtx / 16;
      for (int r = 0; r < 16; r++) {
        const int row = min(r0 + r, N - 1);
        bulk_g2s(dst + r * geo.wrow, W + (int64_t)row * pitch + off, wb, &full[it % STAGES]);
      }
    }
  };
  auto issue_acts = [&](int it) {
    if (it >= n_items || !acts_needed(it)) return;
    const int64_t k0 = (int64_t)(it % geo.items) * geo.units * 256;
    const uint32_t xb = act_bytes(it);
    uint8_t* dst = sm + (size_t)(it % STAGES) * slot_bytes + geo.wbytes;
    for (int b = 0; b < B; b++) {
      bulk_g2s(dst + b * xs_stride, qx + (int64_t)b * K + k0, xb, &full[it % STAGES]);
      bulk_g2s(dst + B * xs_stride + b * (geo.xbytes / 4), ds + (int64_t)b * nblk + (k0 >> 5), xb / 4,
               &full[it % STAGES]);
    }
  };
  // weights do not depend on the previous kernel: their copies go out before the dependency wait
  if (threadIdx.x == 0)
    for (int it = 0; it < STAGES - 1; it++) issue_weights(it);
  pdl_wait();
  if (threadIdx.x == 0)
    for (int it = 0; it < STAGES - 1; it++) issue_acts(it);

  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int it = 0; it < n_items; it++) {
    const int part = it % geo.items;
    tc::mbar_wait(&full[it % STAGES], (it / STAGES) & 1, err);
    if (!(flags & 1)) {  // flags bit 0: stream only (profiling the data path)
      const uint8_t* slot = sm + (size_t)(it % STAGES) * slot_bytes;
      const int8_t* xslot = reinterpret_cast<const int8_t*>(slot + geo.wbytes);
      const float2* dslot = reinterpret_cast<const float2*>(slot + geo.wbytes + B * xs_stride);
      const int dstride = geo.xbytes / 32;  // float2 per token row
      const float2* d0 = dslot + min(2 * t, B - 1) * dstride;
      const float2* d1 = dslot + min(2 * t + 1, B - 1) * dstride;
      const int8_t* xs = xslot + min(g, B - 1) * xs_stride;
      const int u_end = min(geo.units, n_units - part * geo.units);
      for (int u = warp; u < u_end; u += WARPS) {
        const int ug = part * geo.units + u;  // global super unit
        const uint8_t* wa = slot + g * geo.wrow + u * UB;
        const uint8_t* wb = slot + (g + 8) * geo.wrow + u * UB;
        const int nvalid = (int)min((int64_t)8, nblk - (int64_t)ug * 8);
        float a4[4] = {0.f, 0.f, 0.f, 0.f};
        tile_unit<QT>(wa, wb, xs + u * 256, d0 + u * 8, d1 + u * 8, nvalid, g < B, t, a4);
        if (2 * t < B) { acc[0] += a4[0]; acc[2] += a4[2]; }
        if (2 * t + 1 < B) { acc[1] += a4[1]; acc[3] += a4[3]; }
      }
    }
    const bool last = part == geo.items - 1;
    const int rb = (it / geo.items) & 1;
    if (last) {
#pragma unroll
      for (int e = 0; e < 4; e++) red[rb][warp][lane][e] = acc[e];
    }
    __syncthreads();  // ring slot retired; tile partials published
    if (threadIdx.x == 0) {
      issue_weights(it + STAGES - 1);
      issue_acts(it + STAGES - 1);
    }
    if (!last) continue;
    acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
    if (warp != 0) continue;
    float v[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < WARPS; w++) sum += red[rb][w][lane][e];
      v[e] = sum;
    }
    const int r0 = item_tile(it) * 16;
    const int tok0 = 2 * t, tok1 = 2 * t + 1;
    const int rowa = r0 + g, rowb = r0 + g + 8;
    if (epi == EPI_SWIGLU) {
      // tile rows [r0, r0+8) are gate rows of outputs [r0/2, r0/2+8), rows [r0+8, r0+16) the matching up rows
      const int o = (r0 >> 1) + g;
      if (rowb < N) {
        const float bg = bias ? bias[rowa] : 0.f, bu = bias ? bias[rowb] : 0.f;
        if (tok0 < B) y[(int64_t)tok0 * ldy + o] = silu(v[0] + bg) * (v[2] + bu);
        if (tok1 < B) y[(int64_t)tok1 * ldy + o] = silu(v[1] + bg) * (v[3] + bu);
      }
      continue;
    }
#pragma unroll
    for (int half = 0; half < 2; half++) {
      const int row = half ? rowb : rowa;
      if (row >= N) continue;
      const float bv = bias ? bias[row] : 0.f;
      const float v0 = v[2 * half] + bv, v1 = v[2 * half + 1] + bv;
      if (tok0 < B) {
        float* p = y + (int64_t)tok0 * ldy + row;
        *p = epi == EPI_ADD ? *p + v0 : v0;
      }
      if (tok1 < B) {
        float* p = y + (int64_t)tok1 * ldy + row;
        *p = epi == EPI_ADD ? *p + v1 : v1;
      }
    }
  }
  pdl_launch_dependents();
}

// activation quantizer with enough CTAs to fill the GPU: grid (B, ceil(K / 256)); each CTA
// quantizes 8 blocks of 32 and, for the fused RMSNorm, recomputes its row's sum of squares.
// unit != 0: one scale for the CTA's whole 256-column unit (max |v| over the unit / 127), stored in
// each of its eight (scale, sum) entries -- the same format, with the scale uniform over a unit,
// which lets the tile-packed GEMV apply it once per unit instead of once per 32 columns.
__global__ void k_quant_act_wide(const float* __restrict__ x, int64_t ldx, const float* __restrict__ gamma, float eps,
                                 int K, int8_t* __restrict__ qx, float2* __restrict__ ds, const uint8_t* __restrict__ pf,
                                 int64_t pf_bytes, int unit) {
  l2_prefetch(pf, pf_bytes);
  pdl_wait();
  const int b = blockIdx.x;
  const float* xr = x + (int64_t)b * ldx;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float inv = 1.f;
  if (gamma) {
    __shared__ float red[8];
    float ss = 0.f;
    for (int i = threadIdx.x * 4; i < K; i += blockDim.x * 4) {
      float4 v = *reinterpret_cast<const float4*>(xr + i);
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < 8; w++) tot += red[w];
    inv = rsqrtf(tot / (float)K + eps);
  }
  pdl_launch_dependents();
  const int blk = blockIdx.y * 8 + warp;
  const bool live = blk * 32 < K;
  const int i = blk * 32 + lane;
  float v = live ? xr[i] * inv : 0.f;
  if (gamma && live) v *= gamma[i];
  float amax = warp_max(fabsf(v));
  if (unit) {
    __shared__ float umax[8];
    if (lane == 0) umax[warp] = amax;
    __syncthreads();
#pragma unroll
    for (int w = 0; w < 8; w++) amax = fmaxf(amax, umax[w]);
  }
  if (!live) return;
  float d = amax / 127.f;
  const float q = d > 0.f ? rintf(v / d) : 0.f;
  const float s = warp_sum(q) * d;  // sum of the dequantized values (exact integer sum x scale)
  qx[(int64_t)b * K + i] = (int8_t)q;
  if (lane == 0) ds[(int64_t)b * (K / 32) + blk] = make_float2(d, s);
}

}  // namespace

void qmmv(torch::Tensor w, int64_t qtype, int64_t N, int64_t K, int64_t pitch, torch::Tensor qx, torch::Tensor ds,
          int64_t B, torch::Tensor y, c10::optional<torch::Tensor> bias, int64_t epi, int64_t flags) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kUInt8, "w: cuda uint8");
  TORCH_CHECK(qtype == QT_Q8_0 ? K % 64 == 0 : K % 256 == 0, "qmmv: K must be a multiple of 256 (64 for Q8_0)");
  TORCH_CHECK(pitch % 16 == 0 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0, "qmmv: 16-byte row pitch/base");
  TORCH_CHECK(w.numel() >= N * pitch, "qmmv: weight buffer smaller than N*pitch");
  TORCH_CHECK(qx.scalar_type() == torch::kInt8 && qx.is_contiguous() && qx.numel() >= B * K, "qmmv: qx");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(qx.data_ptr()) % 16 == 0, "qmmv: qx alignment");
  TORCH_CHECK(ds.scalar_type() == torch::kFloat32 && ds.is_contiguous() && ds.numel() >= B * K / 16, "qmmv: ds");
  TORCH_CHECK(y.scalar_type() == torch::kFloat32 && y.dim() == 2 && y.stride(1) == 1, "qmmv: y [B, *] f32");
  TORCH_CHECK(B >= 1 && B <= 8, "qmmv: 1 <= B <= 8");
  if (epi == EPI_SWIGLU) TORCH_CHECK(N % 16 == 0, "qmmv: SwiGLU needs 8-row interleaved gate/up blocks");
  TORCH_CHECK(y.size(0) >= B && y.size(1) >= (epi == EPI_SWIGLU ? N / 2 : N), "qmmv: y too small");
  const float* bp = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() >= N, "qmmv: bias");
    bp = bias->data_ptr<float>();
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(WARPS * 32);
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int ub = qtype == QT_Q4_K ? 144 : (qtype == QT_Q6_K ? 210 : 8 * 34);
  const int n_units = (int)((K + 255) / 256);
  const int64_t row_bytes = qtype == QT_Q8_0 ? (K / 32) * 34 : (int64_t)n_units * ub;
  int item_max = (int)(((flags >> 12) & 255) ? ((flags >> 12) & 255) * 1024 : 48 * 1024);  // weight bytes per slot
  ItemGeom geo;
  if (16 * pitch <= item_max) {
    geo.whole = true;
    geo.units = n_units;
    geo.items = 1;
    geo.wrow = (int)pitch;
    geo.wbytes = (int)(16 * pitch);
  } else {
    // chunk of whole super units per row; byte size a multiple of 16 (Q6_K: 8 units = 1680 B)
    const int align_units = qtype == QT_Q6_K ? 8 : 1;
    int u = std::max(align_units, (item_max / 16) / ub / align_units * align_units);
    geo.whole = false;
    geo.units = u;
    geo.items = (n_units + u - 1) / u;
    const int span = u * ub;
    geo.wrow = span + ((144 - span % 128) % 128);  // 16 mod 128
    geo.wbytes = 16 * geo.wrow;
  }
  geo.xbytes = geo.units * 256;
  if (geo.xbytes > K) geo.xbytes = (int)((K + 63) / 64 * 64);
  const size_t slot = (size_t)geo.wbytes + (size_t)B * (geo.xbytes + 32 + geo.xbytes / 4);
  // three slots (two items in flight) when they fit, else two; measured best on B200 for the
  // decode shapes (gate/up, LM head, down)
  int stages = 3 * slot <= 200 * 1024 ? 3 : 2;
  if ((flags >> 4) & 15) stages = (int)((flags >> 4) & 15);  // profiling override: pipeline depth
  const size_t smem = (size_t)stages * slot;
  TORCH_CHECK(smem <= 220 * 1024, "qmmv: shared-memory ring too large (", smem, " B)");
  (void)row_bytes;
  cfg.dynamicSmemBytes = smem;
  static int n_sm = 0;
  if (!n_sm) FAK_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, w.get_device()));
  int per_sm = std::max(1, (int)((227 * 1024) / (smem + 2 * WARPS * 32 * 4 * 4 + 64)));
  if ((flags >> 8) & 15) per_sm = std::min(per_sm, (int)((flags >> 8) & 15));  // profiling override
  const int64_t tiles = (N + 15) / 16;
  cfg.gridDim = dim3((unsigned)std::min<int64_t>(tiles, (int64_t)n_sm * per_sm));
  auto args = [&](auto kern) {
    FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, (const uint8_t*)w.data_ptr<uint8_t>(), (int)N, (int)K, pitch,
                                      (const int8_t*)qx.data_ptr<int8_t>(),
                                      (const float2*)reinterpret_cast<float2*>(ds.data_ptr<float>()), (int)B,
                                      y.data_ptr<float>(), (int64_t)y.stride(0), bp, (int)epi, (int*)nullptr, (int)flags, geo));
  };
#define FAK_QMMV(QTV)                                   \
  {                                                     \
    switch (stages) {                                   \
      case 2: args(k_qmmv<QTV, 2>); break;              \
      case 3: args(k_qmmv<QTV, 3>); break;              \
      case 4: args(k_qmmv<QTV, 4>); break;              \
      case 6: args(k_qmmv<QTV, 6>); break;              \
      default: TORCH_CHECK(false, "qmmv: pipeline depth must be 2, 3, 4 or 6"); \
    }                                                   \
  }
  if (qtype == QT_Q4_K) FAK_QMMV(QT_Q4_K)
  else if (qtype == QT_Q6_K) FAK_QMMV(QT_Q6_K)
  else if (qtype == QT_Q8_0) FAK_QMMV(QT_Q8_0)
#undef FAK_QMMV
  else TORCH_CHECK(false, "qmmv: unsupported qtype ", qtype);
}

void quant_act_wide(torch::Tensor x, c10::optional<torch::Tensor> gamma, double eps, torch::Tensor qx,
                    torch::Tensor ds, c10::optional<torch::Tensor> prefetch, bool unit) {
  const uint8_t* pfp = prefetch.has_value() ? reinterpret_cast<const uint8_t*>(prefetch->data_ptr()) : nullptr;
  const int64_t pfb = prefetch.has_value() ? prefetch->numel() * prefetch->element_size() : 0;
  TORCH_CHECK(x.is_cuda() && x.scalar_type() == torch::kFloat32 && x.dim() == 2 && x.stride(1) == 1, "x: [B,K] f32");
  const int B = (int)x.size(0), K = (int)x.size(1);
  TORCH_CHECK(K % 32 == 0 && x.stride(0) % 4 == 0, "K multiple of 32, row stride multiple of 4");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0, "x alignment");
  TORCH_CHECK(qx.scalar_type() == torch::kInt8 && qx.numel() >= (int64_t)B * K, "qx");
  TORCH_CHECK(ds.scalar_type() == torch::kFloat32 && ds.numel() >= (int64_t)B * K / 16, "ds");
  const float* g = nullptr;
  if (gamma.has_value()) {
    TORCH_CHECK(gamma->numel() == K && gamma->scalar_type() == torch::kFloat32, "gamma");
    g = gamma->data_ptr<float>();
  }
  if (B == 0) return;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(B, (K + 255) / 256);
  cfg.blockDim = dim3(256);
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k_quant_act_wide, (const float*)x.data_ptr<float>(), (int64_t)x.stride(0), g,
                                    (float)eps, K, qx.data_ptr<int8_t>(), reinterpret_cast<float2*>(ds.data_ptr<float>()),
                                    pfp, pfb, unit ? 1 : 0));
}
