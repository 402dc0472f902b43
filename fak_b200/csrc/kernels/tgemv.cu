// Decode GEMV over tile-packed GGML blocks on the integer tensor cores (B <= 8 tokens).
//
// Weight layout ("tile-packed").  Rows are grouped in tiles of 16 and each row's blocks in
// 256-weight super units; the 16 rows x 1 unit of a tile ("unit tile") are stored contiguously,
// split into planes so that every field a thread needs is an aligned, bank-conflict-free shared
// load once the unit tile sits in shared memory:
//   Q4_K  2304 B: hdr [16][16] (d, dmin, 12 scale bytes) | qs [16][128]
//   Q6_K  3360 B: ql [16][128] | qh [16][64] (tile-row order) | scales [16][16] | d [16][2]
//   Q8_0  4352 B: qs [16][256] (8 blocks x 32) | d [16][8][2]
//   G4    2304 B: as Q4_K, the header holding (s0, m0, s1, m1) f32 of the two 128-groups (AWQ / GPTQ)
// Plane row ("slot") s holds tile row (s >> 1) + 8 (s & 1), so the two rows an MMA thread owns
// (g and g + 8) are adjacent slots; the 16-byte chunks of the quant planes are XOR-swizzled by slot
// (Q4_K/Q8_0 qs: chunk ^ (s & 6); Q6_K ql: chunk ^ ((s >> 1) & 7)).  The Q6_K qh plane keeps tile-row
// order (row r at 64 r bytes, so rows g and g+1 sit in opposite halves of the banks) with chunk ^ ((r >> 1) & 3).
// The block bytes themselves are unchanged; only their placement differs from the GGUF rows.
//
// Work decomposition.  A work item is one tile x one K slice and belongs to ONE warp: the warp
// streams its unit tiles through a private ring of shared-memory slots (1-D TMA bulk copies
// completing on per-slot mbarriers, lane 0 as producer), so no CTA-wide barrier sits in the main
// loop.  All warps of a CTA work on the same K slice, whose activations (int8 codes, per-32
// (scale, sum) pairs) are staged once per CTA.  When the matrix has too few tiles to occupy every
// warp, K is split into slices; the slice partials meet in a global scratch and the last warp to
// finish a tile (atomic ticket) sums them in slice order, so results are deterministic and
// independent of the batch size.
//
// Per 32-element sub-block and thread (rows g, g+8; tokens 2t, 2t+1): one m16n8k32 integer MMA
// whose accumulator starts at the float-conversion constant 0x4B400000, so the int32 result read
// as a float is 12582912 + dot exactly (|dot| < 2^22), then
//   Q4_K  acc += (d*sc) * dx * dot - (dmin*m) * sum(xq)    (nibbles via u8 x s8; high nibbles
//                                                           in place, scale pre-divided by 16)
//   Q6_K  acc += (d*sc) * dx * dot16                        (m16n8k16 per 16-element sub-block;
//                                                           the -32 offset enters through the
//                                                           accumulator start: -32 * sum(qx))
//   Q8_0  acc += d * dx * dot
// The per-(row, sub-block) float scales of a unit tile are decoded once per warp into a small
// shared table (each lane decodes 4-8 of them) instead of by every thread that uses them.
// Reference: the per-op GEMV kernels of internal/compute/cuda_kernels.cu (k_q8_matvec and the
// Q4_K/Q6_K dequant paths), which read one row per warp from the GGUF rows.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include "tc.cuh"

using namespace fak;

namespace {

enum Epi : int { EPI_STORE = 0, EPI_ADD = 1, EPI_SWIGLU = 2, EPI_GEGLU = 3, EPI_OAI = 4 };
constexpr int MAXNT = 4;  // n8 token tiles per launch: up to 32 tokens
constexpr int MAGIC_I = 0x4B400000;
constexpr float MAGIC_F = 12582912.0f;

template <int QT> struct Tile;
template <> struct Tile<QT_Q4_K> { static constexpr int UT = 2304; static constexpr int TABF = 16 * 8 * 2; };
template <> struct Tile<QT_G4> { static constexpr int UT = 2304; static constexpr int TABF = 16 * 8 * 2; };   // Q4_K shape
template <> struct Tile<QT_Q6_K> { static constexpr int UT = 3360; static constexpr int TABF = 16 * 16; };
template <> struct Tile<QT_Q8_0> { static constexpr int UT = 4352; static constexpr int TABF = 16 * 8; };

FAK_DEV void mma_u8s8_k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c0, int c1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}
FAK_DEV void mma_s8s8_k32(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1, int c0, int c1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%11,%10,%11};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(c0), "r"(c1));
}
FAK_DEV void mma_u8s8_k16(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t b0, int c0, int c1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%7,%8};"
      : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
      : "r"(a0), "r"(a1), "r"(b0), "r"(c0), "r"(c1));
}
FAK_DEV float magic_f(int c) { return __int_as_float(c) - MAGIC_F; }
// byte i of w as a float (exact), without the XU pipe
FAK_DEV float ubyte_f(uint32_t w, int i) {
  return __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7650 + i) ) - 8388608.0f;
}

FAK_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          tc::smem_addr(dst)),
      "l"(src), "r"(bytes), "r"(tc::smem_addr(bar))
      : "memory");
}

struct TGeo {
  int T;        // 16-row tiles
  int U;        // 256-weight units per row
  int S;        // K slices
  int Us;       // units per slice (last slice may hold fewer)
  int P;        // CTAs per slice
  int xstride;  // shared bytes per token row of activation codes
  int dstride;  // float2 per token row of the staged (scale, sum) pairs
};

// Shared-memory carve-up (byte offsets), identical on host and device.
struct TSmem {
  int ring, xs, dsr, dsT, czT, tab, bars, total;
};
__host__ __device__ inline TSmem tsmem(int qt, int W, int R, int NT, const TGeo& g) {
  const bool q4 = qt == QT_Q4_K || qt == QT_G4;   // G4 (AWQ / GPTQ) tiles have the Q4_K shape
  const int UT = q4 ? 2304 : (qt == QT_Q6_K ? 3360 : 4352);
  const int TABF = q4 ? 256 : (qt == QT_Q6_K ? 256 : 128);
  const int MB = 8 * NT;  // token rows staged
  TSmem s;
  s.ring = 0;
  s.xs = W * R * UT;
  s.dsr = s.xs + MB * g.xstride;
  s.dsT = s.dsr + MB * g.dstride * 8;
  s.czT = s.dsT + g.Us * 8 * MB * 8;
  s.tab = s.czT + (qt == QT_Q6_K ? g.Us * 16 * MB * 4 : 0);
  s.bars = s.tab + W * TABF * 4;
  s.total = s.bars + (W * R + 1) * 8;
  return s;
}

// ---- one unit tile -------------------------------------------------------------------------
// wt: the unit tile in shared memory; tab: this warp's scale table; xr: token g's codes at this
// unit (token 8 nt + g at xr + 8 nt * xstride); dsT: (scale, sum) at this unit's first block,
// [block][token]; czT (Q6_K): accumulator starts at this unit's first 16-block, [k16][token].
// The weight fragments and scales of a sub-block are unpacked once and reused for every n8 tile.
template <int QT, int NT>
FAK_DEV void unit_tile(const uint8_t* __restrict__ wt, float* __restrict__ tab, const int8_t* __restrict__ xr,
                       int xstride, const float2* __restrict__ dsT, const int* __restrict__ czT, int lane,
                       float (&acc)[NT][4]) {
  constexpr int MB = 8 * NT;
  const int g = lane >> 2, t = lane & 3;
  const int sA = 2 * g, sB = 2 * g + 1;
  if constexpr (QT == QT_Q4_K || QT == QT_G4) {
    if constexpr (QT == QT_G4) {  // header (s0, m0, s1, m1): lane -> slot lane>>1, 128-group lane&1 = sub-blocks 4*(lane&1) .. +3
      const int s = lane >> 1, jh = lane & 1;
      const float4 h = *reinterpret_cast<const float4*>(wt + 16 * s);
      const float sc = jh ? h.z : h.x, mn = jh ? h.w : h.y;
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int j = 4 * jh + i;
        reinterpret_cast<float2*>(tab)[j * 16 + s] = make_float2(sc * ((j & 1) ? 0.0625f : 1.0f), mn);
      }
    } else {  // scale table: lane -> slot lane>>1, sub-blocks 4*(lane&1) .. +3
      const int s = lane >> 1, jh = lane & 1;
      const uint4 h = *reinterpret_cast<const uint4*>(wt + 16 * s);
      const float d = __half2float(__ushort_as_half((uint16_t)(h.x & 0xffff)));
      const float dm = __half2float(__ushort_as_half((uint16_t)(h.x >> 16)));
      // 6-bit (scale, min) of sub-blocks 0-3 are the low 6 bits of bytes 0-3 / 4-7; those of
      // sub-blocks 4-7 combine the nibbles of bytes 8-11 with the top 2 bits of bytes 0-7
      const uint32_t scw = jh ? ((h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u)) : (h.y & 0x3F3F3F3Fu);
      const uint32_t mw = jh ? (((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u)) : (h.z & 0x3F3F3F3Fu);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const int j = 4 * jh + i;
        const float a = d * ubyte_f(scw, i) * ((j & 1) ? 0.0625f : 1.0f);  // odd j: high nibbles x16
        reinterpret_cast<float2*>(tab)[j * 16 + s] = make_float2(a, dm * ubyte_f(mw, i));
      }
    }
    __syncwarp();
    const uint8_t* qs = wt + 256;
    const uint8_t* rA = qs + 128 * sA + 8 * (t & 1);
    const uint8_t* rB = qs + 128 * sB + 8 * (t & 1);
#pragma unroll
    for (int c = 0; c < 4; c++) {
      const int q = 2 * c + (t >> 1);
      const uint2 qa = *reinterpret_cast<const uint2*>(rA + 16 * (q ^ (sA & 6)));
      const uint2 qb = *reinterpret_cast<const uint2*>(rB + 16 * (q ^ (sB & 6)));
#pragma unroll
      for (int hi = 0; hi < 2; hi++) {
        const int j = 2 * c + hi;
        const uint32_t m = hi ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
        const uint32_t a[4] = {qa.x & m, qb.x & m, qa.y & m, qb.y & m};
        const float4 am = *reinterpret_cast<const float4*>(tab + 2 * (j * 16 + sA));  // A_g, M_g, A_g8, M_g8
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
          const uint2 xb = *reinterpret_cast<const uint2*>(xr + nt * 8 * xstride + 32 * j + 8 * t);
          int cc[4];
          mma_u8s8_k32(cc, a, xb.x, xb.y, MAGIC_I, MAGIC_I);
          const float4 dx = *reinterpret_cast<const float4*>(dsT + j * MB + nt * 8 + 2 * t);  // d0, s0, d1, s1
          acc[nt][0] = fmaf(am.x * dx.x, magic_f(cc[0]), fmaf(-am.y, dx.y, acc[nt][0]));
          acc[nt][1] = fmaf(am.x * dx.z, magic_f(cc[1]), fmaf(-am.y, dx.w, acc[nt][1]));
          acc[nt][2] = fmaf(am.z * dx.x, magic_f(cc[2]), fmaf(-am.w, dx.y, acc[nt][2]));
          acc[nt][3] = fmaf(am.z * dx.z, magic_f(cc[3]), fmaf(-am.w, dx.w, acc[nt][3]));
        }
      }
    }
  } else if constexpr (QT == QT_Q6_K) {
    {  // scale table: lane -> slot lane>>1, sub-blocks 8*(lane&1) .. +7
      const int s = lane >> 1, sh = lane & 1;
      const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(wt + 3328 + 2 * s)));
      const uint2 sc = *reinterpret_cast<const uint2*>(wt + 3072 + 16 * s + 8 * sh);
#pragma unroll
      for (int i = 0; i < 8; i++) {
        const uint32_t w = i < 4 ? sc.x : sc.y;
        const int v = (int)(int8_t)((w >> (8 * (i & 3))) & 0xff);
        tab[(8 * sh + i) * 16 + s] = d * i2f_exact22(v);
      }
    }
    __syncwarp();
    const uint8_t* ql = wt;
    const uint8_t* qh = wt + 2048;
    const int f8 = g, f4 = (g >> 1) & 3;  // swizzle keys of ql (slots 2g, 2g+1) and qh (rows g, g+8)
#pragma unroll
    for (int n = 0; n < 2; n++) {
#pragma unroll
      for (int h = 0; h < 2; h++) {
        const int c1 = 4 * n + h, c2 = 4 * n + 2 + h, ch = 2 * n + h;
        const uint32_t la0 = *reinterpret_cast<const uint32_t*>(ql + 128 * sA + 16 * (c1 ^ f8) + 4 * t);
        const uint32_t la1 = *reinterpret_cast<const uint32_t*>(ql + 128 * sA + 16 * (c2 ^ f8) + 4 * t);
        const uint32_t lb0 = *reinterpret_cast<const uint32_t*>(ql + 128 * sB + 16 * (c1 ^ f8) + 4 * t);
        const uint32_t lb1 = *reinterpret_cast<const uint32_t*>(ql + 128 * sB + 16 * (c2 ^ f8) + 4 * t);
        const uint32_t ha = *reinterpret_cast<const uint32_t*>(qh + 64 * g + 16 * (ch ^ f4) + 4 * t);
        const uint32_t hb = *reinterpret_cast<const uint32_t*>(qh + 64 * (g + 8) + 16 * (ch ^ f4) + 4 * t);
#pragma unroll
        for (int kk = 0; kk < 4; kk++) {
          const uint32_t la = (kk & 1) ? la1 : la0, lb = (kk & 1) ? lb1 : lb0;
          const int ls = (kk >> 1) * 4, hs = 2 * kk;
          const uint32_t a0 = ((la >> ls) & 0x0F0F0F0Fu) | (((ha >> hs) & 0x03030303u) << 4);
          const uint32_t a1 = ((lb >> ls) & 0x0F0F0F0Fu) | (((hb >> hs) & 0x03030303u) << 4);
          const int e0 = 128 * n + 32 * kk + 16 * h;  // first weight of this 16-block
          const float2 A = *reinterpret_cast<const float2*>(tab + (e0 >> 4) * 16 + sA);
#pragma unroll
          for (int nt = 0; nt < NT; nt++) {
            const uint32_t xv = *reinterpret_cast<const uint32_t*>(xr + nt * 8 * xstride + e0 + 4 * t);
            const int2 cz = *reinterpret_cast<const int2*>(czT + (e0 >> 4) * MB + nt * 8 + 2 * t);
            int cc[4];
            mma_u8s8_k16(cc, a0, a1, xv, cz.x, cz.y);
            const float4 dx = *reinterpret_cast<const float4*>(dsT + (e0 >> 5) * MB + nt * 8 + 2 * t);
            acc[nt][0] = fmaf(A.x * dx.x, magic_f(cc[0]), acc[nt][0]);
            acc[nt][1] = fmaf(A.x * dx.z, magic_f(cc[1]), acc[nt][1]);
            acc[nt][2] = fmaf(A.y * dx.x, magic_f(cc[2]), acc[nt][2]);
            acc[nt][3] = fmaf(A.y * dx.z, magic_f(cc[3]), acc[nt][3]);
          }
        }
      }
    }
  } else {  // Q8_0
    {
      const int s = lane >> 1, bh = lane & 1;
      const uint2 dd = *reinterpret_cast<const uint2*>(wt + 4096 + 16 * s + 8 * bh);
#pragma unroll
      for (int i = 0; i < 4; i++) {
        const uint32_t w = i < 2 ? dd.x : dd.y;
        tab[(4 * bh + i) * 16 + s] = __half2float(__ushort_as_half((uint16_t)(w >> (16 * (i & 1)))));
      }
    }
    __syncwarp();
    const uint8_t* rA = wt + 256 * sA + 8 * (t & 1);
    const uint8_t* rB = wt + 256 * sB + 8 * (t & 1);
#pragma unroll
    for (int b = 0; b < 8; b++) {
      const int q = 2 * b + (t >> 1);
      const uint2 qa = *reinterpret_cast<const uint2*>(rA + 16 * (q ^ (sA & 6)));
      const uint2 qb = *reinterpret_cast<const uint2*>(rB + 16 * (q ^ (sB & 6)));
      const uint32_t a[4] = {qa.x, qb.x, qa.y, qb.y};
      const float2 D = *reinterpret_cast<const float2*>(tab + b * 16 + sA);
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        const uint2 xb = *reinterpret_cast<const uint2*>(xr + nt * 8 * xstride + 32 * b + 8 * t);
        int cc[4];
        mma_s8s8_k32(cc, a, xb.x, xb.y, MAGIC_I, MAGIC_I);
        const float4 dx = *reinterpret_cast<const float4*>(dsT + b * MB + nt * 8 + 2 * t);
        acc[nt][0] = fmaf(D.x * dx.x, magic_f(cc[0]), acc[nt][0]);
        acc[nt][1] = fmaf(D.x * dx.z, magic_f(cc[1]), acc[nt][1]);
        acc[nt][2] = fmaf(D.y * dx.x, magic_f(cc[2]), acc[nt][2]);
        acc[nt][3] = fmaf(D.y * dx.z, magic_f(cc[3]), acc[nt][3]);
      }
    }
  }
  __syncwarp();  // table and slot reads done before the next unit overwrites them
}

// ---- one Q4_K unit tile, activations with one scale per 256-column unit ("unit scale") ---------
// The per-sub-block scales are integers (6 bits), so with a single activation scale dx per unit the
// dot product of a row with a token is
//   dx * ( d * sum_j sc_j * dot_j  -  dmin * sum_j m_j * s_j )
// where dot_j = sum of code products of sub-block j (one m16n8k32 integer MMA) and s_j = sum of the
// token's codes in sub-block j.  The first sum runs in int32 registers (one IMAD per MMA value; high
// nibbles stay in place, so their products carry a factor 16 that one exact shift removes), the
// second is four dp2a per (row, token) over 16-bit packed s_j -- one float conversion and three
// float operations per value per unit, instead of four float operations per value per sub-block.
// dxu: this unit's scale per staged token; s16: this unit's packed sums, [token][4] x (s_2i | s_2i+1 << 16).
template <int NT>
FAK_DEV void unit_tile_q4k_us(const uint8_t* __restrict__ wt, const int8_t* __restrict__ xr, int xstride,
                              const float* __restrict__ dxu, const int* __restrict__ s16, int lane,
                              float (&acc)[NT][4]) {
  const int g = lane >> 2, t = lane & 3;
  const int sA = 2 * g, sB = 2 * g + 1;
  const uint4 hA = *reinterpret_cast<const uint4*>(wt + 16 * sA);
  const uint4 hB = *reinterpret_cast<const uint4*>(wt + 16 * sB);
  // 6-bit (scale, min) bytes of sub-blocks 0-3 (low 6 bits of header bytes 0-3 / 4-7) and 4-7
  // (nibbles of bytes 8-11 with the top 2 bits of bytes 0-7)
  const uint32_t scA0 = hA.y & 0x3F3F3F3Fu, mA0 = hA.z & 0x3F3F3F3Fu;
  const uint32_t scA1 = (hA.w & 0x0F0F0F0Fu) | ((hA.y >> 2) & 0x30303030u);
  const uint32_t mA1 = ((hA.w >> 4) & 0x0F0F0F0Fu) | ((hA.z >> 2) & 0x30303030u);
  const uint32_t scB0 = hB.y & 0x3F3F3F3Fu, mB0 = hB.z & 0x3F3F3F3Fu;
  const uint32_t scB1 = (hB.w & 0x0F0F0F0Fu) | ((hB.y >> 2) & 0x30303030u);
  const uint32_t mB1 = ((hB.w >> 4) & 0x0F0F0F0Fu) | ((hB.z >> 2) & 0x30303030u);
  int ilo[NT][4], ihi[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; nt++)
#pragma unroll
    for (int v = 0; v < 4; v++) ilo[nt][v] = ihi[nt][v] = 0;
  const uint8_t* qs = wt + 256;
  const uint8_t* rA = qs + 128 * sA + 8 * (t & 1);
  const uint8_t* rB = qs + 128 * sB + 8 * (t & 1);
#pragma unroll
  for (int c = 0; c < 4; c++) {
    const int q = 2 * c + (t >> 1);
    const uint2 qa = *reinterpret_cast<const uint2*>(rA + 16 * (q ^ (sA & 6)));
    const uint2 qb = *reinterpret_cast<const uint2*>(rB + 16 * (q ^ (sB & 6)));
#pragma unroll
    for (int hi = 0; hi < 2; hi++) {
      const int j = 2 * c + hi;
      const uint32_t m = hi ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
      const uint32_t a[4] = {qa.x & m, qb.x & m, qa.y & m, qb.y & m};
      const int sa = (int)(((j < 4 ? scA0 : scA1) >> (8 * (j & 3))) & 0xffu);
      const int sb = (int)(((j < 4 ? scB0 : scB1) >> (8 * (j & 3))) & 0xffu);
#pragma unroll
      for (int nt = 0; nt < NT; nt++) {
        const uint2 xb = *reinterpret_cast<const uint2*>(xr + nt * 8 * xstride + 32 * j + 8 * t);
        int cc[4];
        mma_u8s8_k32(cc, a, xb.x, xb.y, 0, 0);
        int(&I)[4] = hi ? ihi[nt] : ilo[nt];
        I[0] += sa * cc[0];
        I[1] += sa * cc[1];
        I[2] += sb * cc[2];
        I[3] += sb * cc[3];
      }
    }
  }
  const float dA = __half2float(__ushort_as_half((uint16_t)(hA.x & 0xffff)));
  const float dmA = __half2float(__ushort_as_half((uint16_t)(hA.x >> 16)));
  const float dB = __half2float(__ushort_as_half((uint16_t)(hB.x & 0xffff)));
  const float dmB = __half2float(__ushort_as_half((uint16_t)(hB.x >> 16)));
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const int k0 = nt * 8 + 2 * t;
    const int4 p0 = *reinterpret_cast<const int4*>(s16 + 4 * k0);
    const int4 p1 = *reinterpret_cast<const int4*>(s16 + 4 * (k0 + 1));
    const float2 dx = *reinterpret_cast<const float2*>(dxu + k0);
    const int mA_0 = __dp2a_hi(p0.w, (int)mA1, __dp2a_lo(p0.z, (int)mA1, __dp2a_hi(p0.y, (int)mA0, __dp2a_lo(p0.x, (int)mA0, 0))));
    const int mA_1 = __dp2a_hi(p1.w, (int)mA1, __dp2a_lo(p1.z, (int)mA1, __dp2a_hi(p1.y, (int)mA0, __dp2a_lo(p1.x, (int)mA0, 0))));
    const int mB_0 = __dp2a_hi(p0.w, (int)mB1, __dp2a_lo(p0.z, (int)mB1, __dp2a_hi(p0.y, (int)mB0, __dp2a_lo(p0.x, (int)mB0, 0))));
    const int mB_1 = __dp2a_hi(p1.w, (int)mB1, __dp2a_lo(p1.z, (int)mB1, __dp2a_hi(p1.y, (int)mB0, __dp2a_lo(p1.x, (int)mB0, 0))));
    const float v0 = (float)(ilo[nt][0] + (ihi[nt][0] >> 4)), v1 = (float)(ilo[nt][1] + (ihi[nt][1] >> 4));
    const float v2 = (float)(ilo[nt][2] + (ihi[nt][2] >> 4)), v3 = (float)(ilo[nt][3] + (ihi[nt][3] >> 4));
    acc[nt][0] = fmaf(dx.x, fmaf(dA, v0, -dmA * (float)mA_0), acc[nt][0]);
    acc[nt][1] = fmaf(dx.y, fmaf(dA, v1, -dmA * (float)mA_1), acc[nt][1]);
    acc[nt][2] = fmaf(dx.x, fmaf(dB, v2, -dmB * (float)mB_0), acc[nt][2]);
    acc[nt][3] = fmaf(dx.y, fmaf(dB, v3, -dmB * (float)mB_1), acc[nt][3]);
  }
}

// ---- one Q6_K unit tile with unit-scale activations ------------------------------------------
// w = d * sc_j * (q - 32) with signed 8-bit sc_j per 16-element sub-block, so a row's dot product with
// a token is dx * d * sum_j sc_j * dot'_j, where dot'_j = sum (q - 32) x over sub-block j comes out of
// one m16n8k16 integer MMA whose accumulator starts at -32 * (sum of the token's 16 codes): one IMAD
// per MMA value, one conversion and two float operations per value per unit.
// cz: this unit's accumulator starts, [16 sub-blocks][staged tokens].
template <int NT>
FAK_DEV void unit_tile_q6k_us(const uint8_t* __restrict__ wt, const int8_t* __restrict__ xr, int xstride,
                              const float* __restrict__ dxu, const int* __restrict__ cz, int lane,
                              float (&acc)[NT][4]) {
  constexpr int MB = 8 * NT;
  const int g = lane >> 2, t = lane & 3;
  const int sA = 2 * g, sB = 2 * g + 1;
  const uint4 scA = *reinterpret_cast<const uint4*>(wt + 3072 + 16 * sA);
  const uint4 scB = *reinterpret_cast<const uint4*>(wt + 3072 + 16 * sB);
  const uint32_t scAw[4] = {scA.x, scA.y, scA.z, scA.w}, scBw[4] = {scB.x, scB.y, scB.z, scB.w};
  int I[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) I[nt][0] = I[nt][1] = I[nt][2] = I[nt][3] = 0;
  const uint8_t* ql = wt;
  const uint8_t* qh = wt + 2048;
  const int f8 = g, f4 = (g >> 1) & 3;
#pragma unroll
  for (int n = 0; n < 2; n++) {
#pragma unroll
    for (int h = 0; h < 2; h++) {
      const int c1 = 4 * n + h, c2 = 4 * n + 2 + h, ch = 2 * n + h;
      const uint32_t la0 = *reinterpret_cast<const uint32_t*>(ql + 128 * sA + 16 * (c1 ^ f8) + 4 * t);
      const uint32_t la1 = *reinterpret_cast<const uint32_t*>(ql + 128 * sA + 16 * (c2 ^ f8) + 4 * t);
      const uint32_t lb0 = *reinterpret_cast<const uint32_t*>(ql + 128 * sB + 16 * (c1 ^ f8) + 4 * t);
      const uint32_t lb1 = *reinterpret_cast<const uint32_t*>(ql + 128 * sB + 16 * (c2 ^ f8) + 4 * t);
      const uint32_t ha = *reinterpret_cast<const uint32_t*>(qh + 64 * g + 16 * (ch ^ f4) + 4 * t);
      const uint32_t hb = *reinterpret_cast<const uint32_t*>(qh + 64 * (g + 8) + 16 * (ch ^ f4) + 4 * t);
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        const uint32_t la = (kk & 1) ? la1 : la0, lb = (kk & 1) ? lb1 : lb0;
        const int ls = (kk >> 1) * 4, hs = 2 * kk;
        const uint32_t a0 = ((la >> ls) & 0x0F0F0F0Fu) | (((ha >> hs) & 0x03030303u) << 4);
        const uint32_t a1 = ((lb >> ls) & 0x0F0F0F0Fu) | (((hb >> hs) & 0x03030303u) << 4);
        const int e0 = 128 * n + 32 * kk + 16 * h;   // first weight of this 16-block
        const int j = e0 >> 4;                         // sub-block 0..15
        // signed scale bytes: byte j & 3 moved to the top, then an arithmetic shift sign-extends it
        const int sa = (int)(scAw[j >> 2] << (24 - 8 * (j & 3))) >> 24;
        const int sb = (int)(scBw[j >> 2] << (24 - 8 * (j & 3))) >> 24;
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
          const uint32_t xv = *reinterpret_cast<const uint32_t*>(xr + nt * 8 * xstride + e0 + 4 * t);
          const int2 c0 = *reinterpret_cast<const int2*>(cz + j * MB + nt * 8 + 2 * t);
          int cc[4];
          mma_u8s8_k16(cc, a0, a1, xv, c0.x, c0.y);
          I[nt][0] += sa * cc[0];
          I[nt][1] += sa * cc[1];
          I[nt][2] += sb * cc[2];
          I[nt][3] += sb * cc[3];
        }
      }
    }
  }
  const float dA = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(wt + 3328 + 2 * sA)));
  const float dB = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(wt + 3328 + 2 * sB)));
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const float2 dx = *reinterpret_cast<const float2*>(dxu + nt * 8 + 2 * t);
    acc[nt][0] = fmaf(dx.x * dA, (float)I[nt][0], acc[nt][0]);
    acc[nt][1] = fmaf(dx.y * dA, (float)I[nt][1], acc[nt][1]);
    acc[nt][2] = fmaf(dx.x * dB, (float)I[nt][2], acc[nt][2]);
    acc[nt][3] = fmaf(dx.y * dB, (float)I[nt][3], acc[nt][3]);
  }
}

FAK_DEV void epilogue(int tile, const float (&v)[4], int tokb, int lane, int N, int B, float* __restrict__ y,
                      int64_t ldy, const float* __restrict__ bias, int epi) {
  const int g = lane >> 2, t = lane & 3;
  const int r0 = tile * 16, tok0 = tokb + 2 * t, tok1 = tokb + 2 * t + 1;
  const int rowa = r0 + g, rowb = r0 + g + 8;
  if (epi >= EPI_SWIGLU) {
    // rows [r0, r0+8) are the gate rows of outputs [r0/2, r0/2+8), rows [r0+8, r0+16) the up rows
    if (rowb < N) {
      const int o = (r0 >> 1) + g;
      const float bg = bias ? bias[rowa] : 0.f, bu = bias ? bias[rowb] : 0.f;
      if (tok0 < B) y[(int64_t)tok0 * ldy + o] = gated_out(epi, v[0] + bg, v[2] + bu);
      if (tok1 < B) y[(int64_t)tok1 * ldy + o] = gated_out(epi, v[1] + bg, v[3] + bu);
    }
    return;
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

// Tensor-parallel all-reduce fused into the epilogue (K-split row-parallel layers: the attention
// output projection and the down projection).  The warp that finishes a tile pushes its partial into
// slot [parity][me][tile] of every rank's symmetric buffer, sums the W slots of its own buffer in rank
// order -- every rank computes bit-identical values -- and adds the sum to the residual.
//
// Flags travel inside the data (the low-latency line format NCCL calls LL): a lane's four partial
// values go out as two 16-byte stores {v0, epoch, v1, epoch}, {v2, epoch, v3, epoch}, and a reader
// polls its own copy of the line until both epoch words of both halves match.  An aligned 8-byte
// half of a vector store arrives whole, so a matching epoch word vouches for the value beside it:
// there is no separate flag, no system-scope fence and no acquire -- one NVLink write latency per
// tile instead of a fence drain plus a flag round trip (the fence version cost 17 us per projection
// at two ranks against 7 us for the GEMV alone).  The price is twice the bytes on the link, a few
// KB per tile.
//
// Epochs count launches per tile in local memory, so the kernel replays inside CUDA graphs; the
// slots alternate between two halves by epoch parity, so a fast rank's next launch (the next
// projection sharing the slots) cannot overwrite a line a slow rank has not read yet: to write epoch
// e + 2 it must have read every rank's epoch e + 1 lines, which a rank writes only after its launch
// of epoch e (and so its reads of epoch e) finished.  A wait gives up after ``spin`` polls (a launch
// argument) and records error code 4.  No multicast, no TMA from peer memory: peer memory is touched
// by ordinary stores only.
constexpr int AR_MAX_W = 8;
constexpr uint32_t kArSpinLimit = 1u << 24;
struct ArPeers {
  uint8_t* base[AR_MAX_W];  // symmetric buffer base of every rank (W = 0: no all-reduce)
  int W, me;
  int64_t parts_off;        // line slots: [2 parities][AR_MAX_W][T][4 n8 tiles][32 lanes][2] uint4
  uint32_t* epochs;         // local [T]
  uint32_t spin;            // polls of a line before the wait gives up
};

// bytes of the line slots for T tiles
__host__ __device__ constexpr int64_t ar_slot_bytes(int64_t T) { return 2LL * AR_MAX_W * T * 4 * 32 * 32; }

FAK_DEV void ll_store(uint4* p, uint4 v) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
FAK_DEV uint4 ll_load(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

// lane's two lines of (source rank r, tile, n8 tile nt) in the half of epoch ep
FAK_DEV uint4* ar_line(const ArPeers& ar, int owner, int T, uint32_t ep, int r, int tile, int nt, int lane) {
  const int64_t half = (int64_t)(ep & 1u) * AR_MAX_W * T * 4 * 32 * 2;
  return reinterpret_cast<uint4*>(ar.base[owner] + ar.parts_off) + half +
         ((((int64_t)r * T + tile) * 4 + nt) * 32 + lane) * 2;
}

// A warp pushes the final partial of every tile it completes (ar_push) and reads the other ranks'
// lines for those tiles only after AR_PEND of them (or its last tile), so the NVLink latencies of a
// warp's tiles overlap each other and the GEMV of its next tile.  Two pending tiles: a warp rarely
// finalises more (there are more warps than output tiles), and a longer list costs the
// non-all-reduce launches registers they need.
constexpr int AR_PEND = 2;

template <int NT>
FAK_DEV uint32_t ar_push(const ArPeers& ar, int T, int tile, int lane, const float (&v)[NT][4]) {
  uint32_t ep = 0;
  if (lane == 0) ep = ar.epochs[tile] + 1;
  ep = __shfl_sync(0xffffffffu, ep, 0);
#pragma unroll
  for (int nt = 0; nt < NT; nt++) {
    const uint4 l0 = make_uint4(__float_as_uint(v[nt][0]), ep, __float_as_uint(v[nt][1]), ep);
    const uint4 l1 = make_uint4(__float_as_uint(v[nt][2]), ep, __float_as_uint(v[nt][3]), ep);
    for (int r = 0; r < ar.W; r++) {
      uint4* dst = ar_line(ar, r, T, ep, ar.me, tile, nt, lane);
      ll_store(dst, l0);
      ll_store(dst + 1, l1);
    }
  }
  return ep;
}

template <int NT>
FAK_DEV void ar_finish(const ArPeers& ar, int T, const int (&pend)[AR_PEND], const uint32_t (&peps)[AR_PEND], int np,
                       int lane, int N, int B, float* __restrict__ y, int64_t ldy, const float* __restrict__ bias,
                       int epi, int* err) {
#pragma unroll
  for (int i = 0; i < AR_PEND; i++) {
    if (i >= np) break;
    const int tile = pend[i];
    const uint32_t ep = peps[i];
#pragma unroll
    for (int nt = 0; nt < NT; nt++) {
      float v[4] = {0.f, 0.f, 0.f, 0.f};
      // RP ranks' lines in flight at a time (two; one for wider token tiles: registers), each
      // polled until both its lines carry this epoch, then added in rank order
      constexpr int RP = NT == 1 ? 2 : 1;
      for (int r0 = 0; r0 < ar.W; r0 += RP) {
        const int nr = min(RP, ar.W - r0);
        const uint4* src[RP];
        uint4 l[RP][2];
#pragma unroll
        for (int j = 0; j < RP; j++) {
          src[j] = ar_line(ar, ar.me, T, ep, j < nr ? r0 + j : r0, tile, nt, lane);
          l[j][0] = ll_load(src[j]);
          l[j][1] = ll_load(src[j] + 1);
        }
        auto ready = [&]() {
          bool ok = true;
#pragma unroll
          for (int j = 0; j < RP; j++)
            ok = ok && l[j][0].y == ep && l[j][0].w == ep && l[j][1].y == ep && l[j][1].w == ep;
          return ok;
        };
        uint32_t it = 0;
        while (!ready()) {
          if (++it > ar.spin) {
            report_error(err, 4);
            break;
          }
#pragma unroll
          for (int j = 0; j < RP; j++) {
            l[j][0] = ll_load(src[j]);
            l[j][1] = ll_load(src[j] + 1);
          }
        }
#pragma unroll
        for (int j = 0; j < RP; j++)
          if (j < nr) {
            v[0] += __uint_as_float(l[j][0].x); v[1] += __uint_as_float(l[j][0].z);
            v[2] += __uint_as_float(l[j][1].x); v[3] += __uint_as_float(l[j][1].z);
          }
      }
      epilogue(tile, v, 8 * nt, lane, N, B, y, ldy, bias, epi);
    }
    if (lane == 0) ar.epochs[tile] = ep;
  }
}

// One GEMV launch's arguments (a kernel parameter: read from the constant bank, never copied).
struct TgArgs {
  const uint8_t* Wt;     // tile-packed weights
  int N, K;
  const int8_t* qx;      // quantized activations [B, K] and their (scale, sum) pairs, or
  const float2* ds;
  const float* xf;       // fp32 activations [B, ldx] (normalised with gamma when given)
  int64_t ldx;
  const float* gamma;
  float eps;
  int B;
  float* y;              // output [B, ldy]
  int64_t ldy;
  const float* bias;
  int epi;
  float* part;           // split-K partials and tickets
  int* cnt;
  int* err;
  TGeo geo;
  ArPeers ar;
  const uint8_t* pf;     // L2 prefetch of the next kernel's weights
  int64_t pf_bytes;
};

// The GEMV of one CTA (index bid among the geo.P * geo.S CTAs of this matrix).
template <int QT, int W, int R, int NT, bool US>
FAK_DEV void tgemv_cta(const int bid, const TgArgs& a) {
  const uint8_t* __restrict__ Wt = a.Wt;
  const int N = a.N, K = a.K;
  const int8_t* __restrict__ qx = a.qx;
  const float2* __restrict__ ds = a.ds;
  const float* __restrict__ xf = a.xf;
  const int64_t ldx = a.ldx;
  const float* __restrict__ gamma = a.gamma;
  const float eps = a.eps;
  const int B = a.B;
  float* __restrict__ y = a.y;
  const int64_t ldy = a.ldy;
  const float* __restrict__ bias = a.bias;
  const int epi = a.epi;
  float* __restrict__ part = a.part;
  int* __restrict__ cnt = a.cnt;
  int* __restrict__ err = a.err;
  const TGeo& geo = a.geo;
  const ArPeers& ar = a.ar;
  constexpr int UT = Tile<QT>::UT;
  constexpr int TABF = Tile<QT>::TABF;
  constexpr int MB = 8 * NT;  // token rows staged
  extern __shared__ __align__(128) uint8_t sm[];
  const TSmem L = tsmem(QT, W, R, NT, geo);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int slice = bid % geo.S, cta = bid / geo.S;
  const int u0 = slice * geo.Us;
  const int nu = min(geo.Us, geo.U - u0);          // units of this slice
  const int k0 = u0 * 256;
  const int kb = min(nu * 256, K - k0);            // valid activation columns of the slice
  int8_t* xs = reinterpret_cast<int8_t*>(sm + L.xs);
  float2* dsr = reinterpret_cast<float2*>(sm + L.dsr);
  float2* dsT = reinterpret_cast<float2*>(sm + L.dsT);
  int* czT = reinterpret_cast<int*>(sm + L.czT);
  float* tab = reinterpret_cast<float*>(sm + L.tab) + warp * TABF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint64_t* bar = bars + warp * R;
  uint64_t* act_bar = bars + W * R;
  uint8_t* ring = sm + L.ring + (size_t)warp * R * UT;

  const int wg = cta * W + warp, wstride = geo.P * W;
  const int n_my = wg < geo.T ? (geo.T - 1 - wg) / wstride + 1 : 0;
  const int Q = n_my * nu;

  if (lane == 0) {
    for (int i = 0; i < R; i++) tc::mbar_init(&bar[i], 1);
    if (warp == 0) tc::mbar_init(act_bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  // producer state (lane 0): unit tiles are issued in consumption order, R-1 ahead
  int pq = 0, pslot = 0, pu = 0;
  const uint8_t* psrc = Wt + ((int64_t)wg * geo.U + u0) * UT;
  const int64_t next_tile = ((int64_t)wstride * geo.U - nu) * UT;
  auto issue_next = [&]() {
    if (pq >= Q) return;
    tc::mbar_arrive_expect_tx(&bar[pslot], UT);
    bulk_g2s(ring + pslot * UT, psrc, UT, &bar[pslot]);
    pq++;
    pslot = pslot + 1 == R ? 0 : pslot + 1;
    psrc += UT;
    if (++pu == nu) {
      pu = 0;
      psrc += next_tile;
    }
  };
  // weights do not depend on the previous kernel: their first copies go out before the wait
  if (lane == 0)
    for (int i = 0; i < R - 1; i++) issue_next();
  l2_prefetch(a.pf, a.pf_bytes);
  pdl_wait();
  if (xf != nullptr) {
    // fp32 activations: optional RMSNorm (statistics over the whole row), then int8 per 32-block
    // with (scale, sum of the dequantized block) -- the activation quantizer, done while the weight copies fly
    __shared__ float s_inv[8 * MAXNT];
    if (gamma != nullptr) {
      for (int b = warp; b < B; b += W) {
        const float* xr = xf + (int64_t)b * ldx;
        float ss = 0.f;
        for (int i = lane * 4; i < K; i += 128) {
          const float4 v = *reinterpret_cast<const float4*>(xr + i);
          ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        ss = warp_sum(ss);
        if (lane == 0) s_inv[b] = rsqrtf(ss / (float)K + eps);
      }
      __syncthreads();
    }
    const int nblk = nu * 8;
    for (int i = threadIdx.x; i < MB * nblk; i += W * 32) {
      const int b = i / nblk, blk = i - b * nblk;
      const int kk = blk * 32;
      uint32_t w[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
      float2 dsv = make_float2(0.f, 0.f);
      if (b < B && kk < kb) {
        const float* src = xf + (int64_t)b * ldx + k0 + kk;
        const float inv = gamma != nullptr ? s_inv[b] : 1.f;
        float v[32];
#pragma unroll
        for (int j = 0; j < 8; j++) {
          const float4 f = *reinterpret_cast<const float4*>(src + 4 * j);
          float4 gm = make_float4(1.f, 1.f, 1.f, 1.f);
          if (gamma != nullptr) gm = *reinterpret_cast<const float4*>(gamma + k0 + kk + 4 * j);
          v[4 * j] = f.x * inv * gm.x;
          v[4 * j + 1] = f.y * inv * gm.y;
          v[4 * j + 2] = f.z * inv * gm.z;
          v[4 * j + 3] = f.w * inv * gm.w;
        }
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 32; j++) amax = fmaxf(amax, fabsf(v[j]));
        const float d = amax / 127.f;
        const float id = d > 0.f ? 1.f / d : 0.f;
        int isum = 0;
#pragma unroll
        for (int j = 0; j < 32; j++) {
          const int qc = (int)rintf(v[j] * id);
          isum += qc;
          w[j >> 2] |= ((uint32_t)qc & 0xffu) << (8 * (j & 3));
        }
        dsv = make_float2(d, (float)isum * d);  // sum of the dequantized values
      }
      uint4* dst = reinterpret_cast<uint4*>(xs + b * geo.xstride + kk);
      dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
      dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
      dsT[blk * MB + b] = dsv;
    }
  } else {
    if (threadIdx.x == 0) {
      const uint32_t dsb = (uint32_t)(kb / 4);  // (scale, sum) bytes of the slice per token
      tc::mbar_arrive_expect_tx(act_bar, (uint32_t)B * ((uint32_t)kb + dsb));
      for (int b = 0; b < B; b++) {
        bulk_g2s(xs + b * geo.xstride, qx + (int64_t)b * K + k0, (uint32_t)kb, act_bar);
        bulk_g2s(dsr + b * geo.dstride, ds + (int64_t)b * (K / 32) + k0 / 32, dsb, act_bar);
      }
    }
    // zero the activation columns no copy writes (missing tokens, padding past K)
    for (int i = threadIdx.x; i < MB * (nu * 256 / 16); i += W * 32) {
      const int b = i / (nu * 16), c = (i % (nu * 16)) * 16;
      if (b >= B || c >= kb) *reinterpret_cast<uint4*>(xs + b * geo.xstride + c) = make_uint4(0, 0, 0, 0);
    }
    tc::mbar_wait(act_bar, 0, err);
    if constexpr (US) {
      // unit scale: the unit's scale per token, and the token's code sums per 32-block packed in
      // 16-bit pairs ([unit][token][4]) -- both read by unit_tile_q4k_us
      float* dxu = reinterpret_cast<float*>(dsT);
      int* s16 = reinterpret_cast<int*>(dsT) + nu * MB;
      for (int i = threadIdx.x; i < nu * MB; i += W * 32) {
        const int u = i / MB, b = i % MB;
        dxu[i] = (b < B && u * 256 < kb) ? dsr[b * geo.dstride + u * 8].x : 0.f;
        if constexpr (QT != QT_Q4_K) continue;   // Q6_K: the sub-block sums go into czT below
        const int4* src = reinterpret_cast<const int4*>(xs + b * geo.xstride + u * 256);
        int sum[8];
#pragma unroll
        for (int jb = 0; jb < 8; jb++) {
          const int4 v0 = src[2 * jb], v1 = src[2 * jb + 1];
          int a = __dp4a(v0.x, 0x01010101, 0);
          a = __dp4a(v0.y, 0x01010101, a);
          a = __dp4a(v0.z, 0x01010101, a);
          a = __dp4a(v0.w, 0x01010101, a);
          a = __dp4a(v1.x, 0x01010101, a);
          a = __dp4a(v1.y, 0x01010101, a);
          a = __dp4a(v1.z, 0x01010101, a);
          sum[jb] = __dp4a(v1.w, 0x01010101, a);
        }
        *reinterpret_cast<int4*>(s16 + 4 * i) =
            make_int4((sum[0] & 0xffff) | (sum[1] << 16), (sum[2] & 0xffff) | (sum[3] << 16),
                      (sum[4] & 0xffff) | (sum[5] << 16), (sum[6] & 0xffff) | (sum[7] << 16));
      }
    } else {
      for (int i = threadIdx.x; i < nu * 8 * MB; i += W * 32) {
        const int blk = i / MB, b = i % MB;
        dsT[i] = (b < B && blk * 32 < kb) ? dsr[b * geo.dstride + blk] : make_float2(0.f, 0.f);
      }
    }
  }
  if constexpr (QT == QT_Q6_K) {
    __syncthreads();
    for (int i = threadIdx.x; i < nu * 16 * MB; i += W * 32) {
      const int k16 = i / MB, b = i % MB;
      const int4 v = *reinterpret_cast<const int4*>(xs + b * geo.xstride + 16 * k16);
      int sm4 = __dp4a(v.x, 0x01010101, 0);
      sm4 = __dp4a(v.y, 0x01010101, sm4);
      sm4 = __dp4a(v.z, 0x01010101, sm4);
      sm4 = __dp4a(v.w, 0x01010101, sm4);
      czT[i] = (US ? 0 : MAGIC_I) - 32 * sm4;   // unit scale: plain int32 accumulation
    }
  }
  __syncthreads();

  float acc[NT][4];
#pragma unroll
  for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
  const int g = lane >> 2;
  const int8_t* xg = xs + g * geo.xstride;
  int cslot = 0, ul = 0, tile = wg;
  uint32_t phase = 0;
  int pend[AR_PEND], npend = 0;   // fused all-reduce: tiles pushed, not yet summed
  uint32_t peps[AR_PEND];
  for (int q = 0; q < Q; q++) {
    if (lane == 0) issue_next();  // into the slot released at the end of the previous iteration
    tc::mbar_wait(&bar[cslot], phase, err);
    if constexpr (US && QT == QT_Q4_K)
      unit_tile_q4k_us<NT>(ring + cslot * UT, xg + ul * 256, geo.xstride,
                           reinterpret_cast<const float*>(dsT) + ul * MB,
                           reinterpret_cast<const int*>(dsT) + nu * MB + 4 * ul * MB, lane, acc);
    else if constexpr (US && QT == QT_Q6_K)
      unit_tile_q6k_us<NT>(ring + cslot * UT, xg + ul * 256, geo.xstride,
                           reinterpret_cast<const float*>(dsT) + ul * MB, czT + ul * 16 * MB, lane, acc);
    else
      unit_tile<QT, NT>(ring + cslot * UT, tab, xg + ul * 256, geo.xstride, dsT + ul * 8 * MB,
                        QT == QT_Q6_K ? czT + ul * 16 * MB : nullptr, lane, acc);
    if (++cslot == R) {
      cslot = 0;
      phase ^= 1u;
    }
    if (++ul < nu) continue;
    ul = 0;
    bool have = true;  // this warp holds the tile's final (rank-local) value in acc
    if (geo.S > 1) {
      // partials [slice][tile][n8 tile][lane] float4
      float4* mine = reinterpret_cast<float4*>(part + ((size_t)slice * geo.T + tile) * 128 * NT) + lane;
#pragma unroll
      for (int nt = 0; nt < NT; nt++) mine[32 * nt] = make_float4(acc[nt][0], acc[nt][1], acc[nt][2], acc[nt][3]);
      // the warp barrier orders every lane's partial before lane 0's fence, which then covers them
      // all (one fence per warp, not one per lane) ahead of the ticket
      __syncwarp();
      int old = 0;
      if (lane == 0) {
        __threadfence();
        old = atomicAdd(&cnt[tile], 1);
      }
      old = __shfl_sync(0xffffffffu, old, 0);
      have = old == geo.S - 1;
      if (have) {  // last slice of this tile: reduce in slice order
        __threadfence();
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
          float v[4] = {0.f, 0.f, 0.f, 0.f};
          const float4* src = reinterpret_cast<const float4*>(part + (size_t)tile * 128 * NT) + 32 * nt + lane;
          const size_t sstride = (size_t)geo.T * 128 * NT / 4;   // float4s between slices
          // up to SB slices' partials in flight at once (one L2 round trip per SB, a split of fewer
          // slices included), added in slice order; wider token tiles keep fewer in flight (registers)
          constexpr int SB = NT == 1 ? 8 : 4;
          for (int s = 0; s < geo.S; s += SB) {
            float4 p[SB];
#pragma unroll
            for (int u = 0; u < SB; u++)
              if (s + u < geo.S) p[u] = __ldcg(src + (size_t)(s + u) * sstride);
#pragma unroll
            for (int u = 0; u < SB; u++)
              if (s + u < geo.S) {
                v[0] += p[u].x; v[1] += p[u].y; v[2] += p[u].z; v[3] += p[u].w;
              }
          }
          acc[nt][0] = v[0]; acc[nt][1] = v[1]; acc[nt][2] = v[2]; acc[nt][3] = v[3];
        }
        if (lane == 0) cnt[tile] = 0;  // ready for the next launch
      }
    }
    if (have) {
      if (ar.W > 0) {   // fused all-reduce: push now, read / sum / store in batches
        const uint32_t ep = ar_push<NT>(ar, geo.T, tile, lane, acc);
#pragma unroll
        for (int i = 0; i < AR_PEND; i++)
          if (i == npend) { pend[i] = tile; peps[i] = ep; }
        if (++npend == AR_PEND) {
          ar_finish<NT>(ar, geo.T, pend, peps, npend, lane, N, B, y, ldy, bias, epi, err);
          npend = 0;
        }
      } else {
#pragma unroll
        for (int nt = 0; nt < NT; nt++) epilogue(tile, acc[nt], 8 * nt, lane, N, B, y, ldy, bias, epi);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; nt++) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
    tile += wstride;
  }
  if (npend > 0) ar_finish<NT>(ar, geo.T, pend, peps, npend, lane, N, B, y, ldy, bias, epi, err);
}

template <int QT, int W, int R, int NT, bool US = false>
__global__ void __launch_bounds__(W * 32, 1) k_tgemv(const TgArgs a) {
  tgemv_cta<QT, W, R, NT, US>(blockIdx.x, a);
  pdl_launch_dependents();
}

// Two GEMVs over the same activations in one launch (q|k in Q4_K and v in Q6_K, say): CTAs [0, nA)
// run the first, the rest the second, so the two latency chains (activation staging, weight
// copies, split-K tickets) overlap instead of following one another.
template <int QA, int QB, int W, int R, int NT, bool US>
__global__ void __launch_bounds__(W * 32, 1) k_tgemv_pair(const TgArgs a, const TgArgs b, const int nA) {
  if ((int)blockIdx.x < nA) tgemv_cta<QA, W, R, NT, US>(blockIdx.x, a);
  else tgemv_cta<QB, W, R, NT, US>(blockIdx.x - nA, b);
  pdl_launch_dependents();
}

// ---- grouped expert GEMV (MoE decode) ------------------------------------------------------
// The experts of a layer are stacked row-wise and tile-packed (expert e owns tiles
// [e * Te, (e + 1) * Te)).  A CTA takes one chunk of <= 8 (token, expert) pairs of one expert
// (from the deterministic grouping kernel), gathers their activation rows once, and its warps stream
// every tile of that expert through their private rings (whole K: no split).  Outputs go to the
// pair's row of y: SwiGLU over 8-row interleaved gate/up rows for gate/up, plain store for down.
template <int QT, int W, int R>
__global__ void __launch_bounds__(W * 32, 1)
k_tgemv_moe(const uint8_t* __restrict__ Wt, int Te, int K, const int8_t* __restrict__ qx, const float2* __restrict__ ds,
            int topk, int act_by_token, const int* __restrict__ chunk_expert, const int* __restrict__ chunk_pairs,
            const int* __restrict__ n_chunks, float* __restrict__ y, int64_t ldy, int epi, int* __restrict__ err,
            TGeo geo, const float* __restrict__ bias) {
  constexpr int UT = Tile<QT>::UT;
  constexpr int TABF = Tile<QT>::TABF;
  constexpr int MB = 8;
  extern __shared__ __align__(128) uint8_t sm[];
  const TSmem L = tsmem(QT, W, R, 1, geo);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunk = blockIdx.x;
  pdl_wait();
  if (chunk >= n_chunks[0]) return;
  const int e = chunk_expert[chunk];
  int pr[MB];
#pragma unroll
  for (int s = 0; s < MB; s++) pr[s] = chunk_pairs[chunk * MB + s];
  const int nu = geo.U, kb = K;
  int8_t* xs = reinterpret_cast<int8_t*>(sm + L.xs);
  float2* dsr = reinterpret_cast<float2*>(sm + L.dsr);
  float2* dsT = reinterpret_cast<float2*>(sm + L.dsT);
  int* czT = reinterpret_cast<int*>(sm + L.czT);
  float* tab = reinterpret_cast<float*>(sm + L.tab) + warp * TABF;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.bars);
  uint64_t* bar = bars + warp * R;
  uint64_t* act_bar = bars + W * R;
  uint8_t* ring = sm + L.ring + (size_t)warp * R * UT;
  const int n_my = warp < Te ? (Te - 1 - warp) / W + 1 : 0;
  const int Q = n_my * nu;
  if (lane == 0) {
    for (int i = 0; i < R; i++) tc::mbar_init(&bar[i], 1);
    if (warp == 0) tc::mbar_init(act_bar, 1);
    tc::fence_mbar_init();
  }
  __syncthreads();
  int pq = 0, pslot = 0, pu = 0;
  const uint8_t* psrc = Wt + ((int64_t)e * Te + warp) * nu * UT;
  const int64_t next_tile = ((int64_t)W * nu - nu) * UT;
  auto issue_next = [&]() {
    if (pq >= Q) return;
    tc::mbar_arrive_expect_tx(&bar[pslot], UT);
    bulk_g2s(ring + pslot * UT, psrc, UT, &bar[pslot]);
    pq++;
    pslot = pslot + 1 == R ? 0 : pslot + 1;
    psrc += UT;
    if (++pu == nu) {
      pu = 0;
      psrc += next_tile;
    }
  };
  if (lane == 0)
    for (int i = 0; i < R - 1; i++) issue_next();
  if (threadIdx.x == 0) {
    uint32_t nv = 0;
    for (int s = 0; s < MB; s++) nv += pr[s] >= 0;
    tc::mbar_arrive_expect_tx(act_bar, nv * ((uint32_t)K + (uint32_t)K / 4));
    for (int s = 0; s < MB; s++) {
      if (pr[s] < 0) continue;
      const int64_t row = act_by_token ? pr[s] / topk : pr[s];
      bulk_g2s(xs + s * geo.xstride, qx + row * K, (uint32_t)K, act_bar);
      bulk_g2s(dsr + s * geo.dstride, ds + row * (K / 32), (uint32_t)(K / 4), act_bar);
    }
  }
  for (int i = threadIdx.x; i < MB * (nu * 256 / 16); i += W * 32) {
    const int b = i / (nu * 16), c = (i % (nu * 16)) * 16;
    if (pr[b] < 0 || c >= kb) *reinterpret_cast<uint4*>(xs + b * geo.xstride + c) = make_uint4(0, 0, 0, 0);
  }
  tc::mbar_wait(act_bar, 0, err);
  for (int i = threadIdx.x; i < nu * 8 * MB; i += W * 32) {
    const int blk = i / MB, b = i % MB;
    dsT[i] = (pr[b] >= 0 && blk * 32 < kb) ? dsr[b * geo.dstride + blk] : make_float2(0.f, 0.f);
  }
  if constexpr (QT == QT_Q6_K) {
    __syncthreads();
    for (int i = threadIdx.x; i < nu * 16 * MB; i += W * 32) {
      const int k16 = i / MB, b = i % MB;
      const int4 v = *reinterpret_cast<const int4*>(xs + b * geo.xstride + 16 * k16);
      int sm4 = __dp4a(v.x, 0x01010101, 0);
      sm4 = __dp4a(v.y, 0x01010101, sm4);
      sm4 = __dp4a(v.z, 0x01010101, sm4);
      sm4 = __dp4a(v.w, 0x01010101, sm4);
      czT[i] = MAGIC_I - 32 * sm4;
    }
  }
  __syncthreads();
  float acc[1][4] = {{0.f, 0.f, 0.f, 0.f}};
  const int g = lane >> 2, t = lane & 3;
  const int8_t* xg = xs + g * geo.xstride;
  int cslot = 0, ul = 0, tile = warp;
  uint32_t phase = 0;
  for (int q = 0; q < Q; q++) {
    if (lane == 0) issue_next();
    tc::mbar_wait(&bar[cslot], phase, err);
    unit_tile<QT, 1>(ring + cslot * UT, tab, xg + ul * 256, geo.xstride, dsT + ul * 8 * MB,
                     QT == QT_Q6_K ? czT + ul * 16 * MB : nullptr, lane, acc);
    if (++cslot == R) {
      cslot = 0;
      phase ^= 1u;
    }
    if (++ul < nu) continue;
    ul = 0;
    const int r0 = tile * 16;
    const int p0 = pr[2 * t], p1 = pr[2 * t + 1];
    // per-expert bias (rows of this expert, in the same interleaved order as its weight rows)
    const float* eb = bias ? bias + (int64_t)e * Te * 16 : nullptr;
    const float ba = eb ? eb[r0 + g] : 0.f, bb = eb ? eb[r0 + g + 8] : 0.f;
    if (epi >= EPI_SWIGLU) {
      const int o = (r0 >> 1) + g;
      if (p0 >= 0) y[(int64_t)p0 * ldy + o] = gated_out(epi, acc[0][0] + ba, acc[0][2] + bb);
      if (p1 >= 0) y[(int64_t)p1 * ldy + o] = gated_out(epi, acc[0][1] + ba, acc[0][3] + bb);
    } else {
      if (p0 >= 0) {
        y[(int64_t)p0 * ldy + r0 + g] = acc[0][0] + ba;
        y[(int64_t)p0 * ldy + r0 + g + 8] = acc[0][2] + bb;
      }
      if (p1 >= 0) {
        y[(int64_t)p1 * ldy + r0 + g] = acc[0][1] + ba;
        y[(int64_t)p1 * ldy + r0 + g + 8] = acc[0][3] + bb;
      }
    }
    acc[0][0] = acc[0][1] = acc[0][2] = acc[0][3] = 0.f;
    tile += W;
  }
  pdl_launch_dependents();
}

struct Plan {
  int W, R, NT;
  TGeo geo;
  int smem;
};

int tile_bytes(int qt) { return (qt == QT_Q4_K || qt == QT_G4) ? 2304 : (qt == QT_Q6_K ? 3360 : 4352); }

// Choose the K split, then (warps per CTA, ring depth) and the token tile width.  The split
// minimises the unit tiles on the busiest warp (rounds of tiles x units per slice, plus the split-K
// reduction) among splits whose 8-token staging fits in shared memory; it depends only on the
// matrix shape and the GPU -- never on the batch -- so a token reduces in the same order whatever
// batch it runs in.  Wider token tiles (16 / 32 tokens per launch) are used when their staging fits
// with that split; otherwise the batch runs as several launches of the widest tile that fits.
static const int kCand[][2] = {{16, 3}, {16, 2}, {8, 3}};

TGeo make_geo(int qt, int T, int U, int S0, int n_sm) {
  const int Us = (U + S0 - 1) / S0;
  TGeo g;
  g.T = T;
  g.U = U;
  g.S = (U + Us - 1) / Us;
  g.Us = Us;
  g.P = std::max(1, n_sm / g.S);
  // activation rows 32 mod 128 bytes apart (8-byte loads, Q4_K/Q8_0) or 16 mod 128 (4-byte, Q6_K)
  g.xstride = ((Us * 256 + 127) / 128) * 128 + (qt == QT_Q6_K ? 16 : 32);
  g.dstride = Us * 8;
  return g;
}

Plan make_plan(int qt, int64_t N, int64_t K, int NT, int n_sm, int max_smem, int force_w, int force_r,
               int force_s) {
  const int T = (int)((N + 15) / 16);
  const int U = (int)((K + 255) / 256);
  int S = force_s;
  if (!S) {
    // over every (warps, depth) candidate and split; ties keep the fewer slices / wider CTA
    double best_cost = 1e30;
    for (auto& c : kCand) {
      for (int s0 = 1; s0 <= std::min(U, n_sm); s0++) {
        const TGeo g = make_geo(qt, T, U, s0, n_sm);
        if (g.S != s0) continue;  // same split as a smaller s0
        if (tsmem(qt, c[0], c[1], 1, g).total > max_smem) continue;
        const int64_t warps = (int64_t)c[0] * g.P;
        const int64_t rounds = (T + warps - 1) / warps;
        const double cost = (double)rounds * (g.Us + (g.S > 1 ? 1.0 : 0.3));
        if (cost < best_cost - 1e-9) {
          best_cost = cost;
          S = g.S;
        }
      }
    }
    TORCH_CHECK(S, "tgemv: no K split fits in shared memory for K=", K);
  }
  const TGeo g = make_geo(qt, T, U, S, n_sm);
  for (int nt = NT; nt >= 1; nt >>= 1) {
    for (auto& c : kCand) {
      const int W = force_w ? force_w : c[0], R = force_r ? force_r : c[1];
      const TSmem L = tsmem(qt, W, R, nt, g);
      if (L.total <= max_smem) return Plan{W, R, nt, g, L.total};
    }
  }
  TORCH_CHECK(false, "tgemv: no launch configuration fits in shared memory for K=", K);
  return Plan{};
}

}  // namespace

int64_t tgemv_unit_bytes(int64_t qtype) { return tile_bytes((int)qtype); }

// Scratch floats / counters the split-K reduction of this shape needs.
std::vector<int64_t> tgemv_workspace(int64_t qtype, int64_t N, int64_t K, int64_t device) {
  int n_sm = 0, max_smem = 0;
  FAK_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, (int)device));
  FAK_CUDA_CHECK(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, (int)device));
  Plan p = make_plan((int)qtype, N, K, 1, n_sm, max_smem, 0, 0, 0);
  return {p.geo.S > 1 ? (int64_t)p.geo.S * p.geo.T * 128 * MAXNT : 0, p.geo.S > 1 ? (int64_t)p.geo.T : 0, p.geo.S,
          p.W, p.R, p.smem};
}

// w: tile-packed weights (uint8, ceil(N/16) * ceil(K/256) unit tiles); activations either quantized
// (qx [B, K] int8, ds [B, K/32, 2]) or fp32 x [B, K] (optionally RMSNorm'd with gamma, eps);
// y [B, *] f32 (row stride y.stride(0)); part/cnt: split-K scratch (cnt zero-initialised; every
// launch leaves it zero again).  flags: bits 0-4 warps, 5-8 ring depth, 9-16 K slices (overrides).
void tgemv(torch::Tensor w, int64_t qtype, int64_t N, int64_t K, c10::optional<torch::Tensor> qx,
           c10::optional<torch::Tensor> ds, c10::optional<torch::Tensor> x, c10::optional<torch::Tensor> gamma,
           double eps, int64_t B, torch::Tensor y, c10::optional<torch::Tensor> bias, int64_t epi, torch::Tensor part,
           torch::Tensor cnt, c10::optional<torch::Tensor> err, int64_t flags, c10::optional<torch::Tensor> ar_peers,
           int64_t ar_me, int64_t ar_parts_off, c10::optional<torch::Tensor> ar_epochs,
           c10::optional<torch::Tensor> prefetch, int64_t ar_spin_limit, bool unit) {
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kUInt8, "tgemv: w cuda uint8");
  const uint8_t* pfp = prefetch.has_value() ? reinterpret_cast<const uint8_t*>(prefetch->data_ptr()) : nullptr;
  const int64_t pfb = prefetch.has_value() ? prefetch->numel() * prefetch->element_size() : 0;
  ArPeers ar{};
  if (ar_peers.has_value()) {  // fused all-reduce over the ranks' symmetric buffers, then residual add
    auto h = ar_peers->cpu();
    TORCH_CHECK(h.scalar_type() == torch::kInt64 && h.numel() >= 1 && h.numel() <= AR_MAX_W, "tgemv: peers");
    TORCH_CHECK(ar_epochs.has_value() && ar_epochs->scalar_type() == torch::kInt32 &&
                    ar_epochs->numel() >= (N + 15) / 16, "tgemv: all-reduce epochs [tiles] int32");
    TORCH_CHECK(epi == EPI_ADD && ar_parts_off % 16 == 0, "tgemv: all-reduce layout");
    ar.W = (int)h.numel();
    ar.me = (int)ar_me;
    for (int r = 0; r < ar.W; r++) ar.base[r] = reinterpret_cast<uint8_t*>(h.data_ptr<int64_t>()[r]);
    ar.parts_off = ar_parts_off;
    ar.epochs = reinterpret_cast<uint32_t*>(ar_epochs->data_ptr<int>());
    TORCH_CHECK(ar_spin_limit >= 0 && ar_spin_limit <= 0xffffffffll, "tgemv: spin limit");
    ar.spin = ar_spin_limit > 0 ? (uint32_t)ar_spin_limit : kArSpinLimit;
  }
  TORCH_CHECK(qtype == QT_Q4_K || qtype == QT_Q6_K || qtype == QT_Q8_0 || qtype == QT_G4, "tgemv: qtype");
  TORCH_CHECK(K % 64 == 0 && (qtype == QT_Q8_0 || K % 256 == 0), "tgemv: K must be a multiple of 256 (64 for Q8_0)");
  const int64_t T = (N + 15) / 16, U = (K + 255) / 256;
  TORCH_CHECK(w.numel() >= T * U * tile_bytes((int)qtype), "tgemv: weight buffer smaller than the tile-packed size");
  TORCH_CHECK(reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0, "tgemv: weight alignment");
  const int8_t* qp = nullptr;
  const float2* dp = nullptr;
  const float* xp = nullptr;
  const float* gp = nullptr;
  int64_t ldx = 0;
  if (x.has_value()) {  // fp32 activations, normalised (gamma) and quantized inside the kernel
    TORCH_CHECK(x->scalar_type() == torch::kFloat32 && x->dim() == 2 && x->stride(1) == 1 && x->size(0) >= B &&
                    x->size(1) >= K && x->stride(0) % 4 == 0 && reinterpret_cast<uintptr_t>(x->data_ptr()) % 16 == 0,
                "tgemv: x [B, >=K] f32, 16-byte aligned rows");
    xp = x->data_ptr<float>();
    ldx = x->stride(0);
    if (gamma.has_value()) {
      TORCH_CHECK(gamma->scalar_type() == torch::kFloat32 && gamma->numel() >= K &&
                      reinterpret_cast<uintptr_t>(gamma->data_ptr()) % 16 == 0, "tgemv: gamma");
      gp = gamma->data_ptr<float>();
    }
  } else {
    TORCH_CHECK(qx.has_value() && ds.has_value(), "tgemv: give x or (qx, ds)");
    TORCH_CHECK(qx->scalar_type() == torch::kInt8 && qx->is_contiguous() && qx->numel() >= B * K, "tgemv: qx");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(qx->data_ptr()) % 16 == 0, "tgemv: qx alignment");
    TORCH_CHECK(ds->scalar_type() == torch::kFloat32 && ds->is_contiguous() && ds->numel() >= B * K / 16, "tgemv: ds");
    TORCH_CHECK(reinterpret_cast<uintptr_t>(ds->data_ptr()) % 16 == 0, "tgemv: ds alignment");
    qp = qx->data_ptr<int8_t>();
    dp = reinterpret_cast<const float2*>(ds->data_ptr<float>());
  }
  TORCH_CHECK(y.scalar_type() == torch::kFloat32 && y.dim() == 2 && y.stride(1) == 1, "tgemv: y [B, *] f32");
  TORCH_CHECK(B >= 1 && B <= 8 * MAXNT, "tgemv: 1 <= B <= 32");
  const int NT = (int)((B + 7) / 8) <= 1 ? 1 : ((B + 7) / 8 <= 2 ? 2 : 4);
  TORCH_CHECK(epi >= EPI_STORE && epi <= EPI_GEGLU, "tgemv: epilogue");
  if (epi >= EPI_SWIGLU) TORCH_CHECK(N % 16 == 0, "tgemv: gated epilogues need 8-row interleaved gate/up blocks");
  TORCH_CHECK(y.size(0) >= B && y.size(1) >= (epi >= EPI_SWIGLU ? N / 2 : N), "tgemv: y too small");
  const float* bp = nullptr;
  if (bias.has_value()) {
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() >= N, "tgemv: bias");
    bp = bias->data_ptr<float>();
  }
  static int n_sm = 0, max_smem = 0;
  if (!n_sm) {
    FAK_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, w.get_device()));
    FAK_CUDA_CHECK(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, w.get_device()));
  }
  Plan p = make_plan((int)qtype, N, K, NT, n_sm, max_smem, (int)(flags & 31), (int)((flags >> 5) & 15),
                     (int)((flags >> 9) & 255));
  if (p.geo.S > 1) {
    TORCH_CHECK(part.scalar_type() == torch::kFloat32 && part.numel() >= (int64_t)p.geo.S * p.geo.T * 128 * p.NT,
                "tgemv: split-K scratch too small");
    TORCH_CHECK(cnt.scalar_type() == torch::kInt32 && cnt.numel() >= p.geo.T, "tgemv: split-K counters too small");
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(p.W * 32);
  cfg.gridDim = dim3(p.geo.P * p.geo.S);
  cfg.dynamicSmemBytes = p.smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int* ep = err.has_value() ? err->data_ptr<int>() : nullptr;
  // the batch runs as launches of up to 8 * p.NT tokens (one launch unless the wide staging did
  // not fit); each token's arithmetic is the same in every launch shape
  const int chunk = 8 * p.NT;
  TORCH_CHECK(ar.W == 0 || B <= chunk, "tgemv: the fused all-reduce takes one launch of at most ", chunk, " tokens");
  auto go = [&](auto kern) {
    FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, p.smem));
    for (int64_t b0 = 0; b0 < B; b0 += chunk) {
      const int nb = (int)std::min<int64_t>(chunk, B - b0);
      TgArgs a{};
      a.Wt = w.data_ptr<uint8_t>();
      a.N = (int)N;
      a.K = (int)K;
      a.qx = qp ? qp + b0 * K : nullptr;
      a.ds = dp ? dp + b0 * (K / 32) : nullptr;
      a.xf = xp ? xp + b0 * ldx : nullptr;
      a.ldx = ldx;
      a.gamma = gp;
      a.eps = (float)eps;
      a.B = nb;
      a.y = y.data_ptr<float>() + b0 * y.stride(0);
      a.ldy = y.stride(0);
      a.bias = bp;
      a.epi = (int)epi;
      a.part = p.geo.S > 1 ? part.data_ptr<float>() : nullptr;
      a.cnt = p.geo.S > 1 ? cnt.data_ptr<int>() : nullptr;
      a.err = ep;
      a.geo = p.geo;
      a.ar = ar;
      a.pf = b0 == 0 ? pfp : nullptr;
      a.pf_bytes = pfb;
      FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, a));
    }
  };
  // unit-scale activations (one scale per 256 columns, ActQ.unit) on Q4_K / Q6_K weights: integer
  // accumulation of the sub-block scales (unit_tile_q4k_us / unit_tile_q6k_us)
  const bool us = unit && (qtype == QT_Q4_K || qtype == QT_Q6_K) && xp == nullptr;
#define FAK_TG_W(QTV, NTV, USV)                                                   \
  {                                                                               \
    if (p.W == 16 && p.R == 3) go(k_tgemv<QTV, 16, 3, NTV, USV>);                 \
    else if (p.W == 16 && p.R == 2) go(k_tgemv<QTV, 16, 2, NTV, USV>);            \
    else if (p.W == 8 && p.R == 3) go(k_tgemv<QTV, 8, 3, NTV, USV>);              \
    else TORCH_CHECK(false, "tgemv: unsupported (warps, depth) ", p.W, ",", p.R); \
  }
#define FAK_TG_NT(QTV, NTV)                                          \
  {                                                                  \
    if constexpr (QTV == QT_Q4_K || QTV == QT_Q6_K) {                \
      if (us) FAK_TG_W(QTV, NTV, true) else FAK_TG_W(QTV, NTV, false) \
    } else FAK_TG_W(QTV, NTV, false)                                 \
  }
#define FAK_TG(QTV)                     \
  {                                     \
    if (p.NT == 1) FAK_TG_NT(QTV, 1)      \
    else if (p.NT == 2) FAK_TG_NT(QTV, 2) \
    else FAK_TG_NT(QTV, 4)                \
  }
  if (qtype == QT_Q4_K) FAK_TG(QT_Q4_K)
  else if (qtype == QT_G4) FAK_TG(QT_G4)
  else if (qtype == QT_Q6_K) FAK_TG(QT_Q6_K)
  else FAK_TG(QT_Q8_0)
#undef FAK_TG
#undef FAK_TG_NT
#undef FAK_TG_W
}

namespace {
// The CTA split and per-matrix plans of a pair launch: the SMs shared in proportion to the weight
// bytes, both plans with 16 warps and a 3-deep ring (the one pair instantiation).  The K splits
// depend on the shapes only, so a token reduces in the same order in every batch; the batch runs
// as launches of the widest token tile whose staging fits for both matrices.
struct PairPlan {
  bool ok = false;
  int nA = 0;
  Plan a, b;
  int64_t partA = 0, cntA = 0, partB = 0, cntB = 0;   // split-K scratch (floats, tickets) of each
};

PairPlan make_pair_plan(int qa, int64_t Na, int qb, int64_t Nb, int64_t K, int64_t B, int n_sm, int max_smem) {
  PairPlan pp;
  if (!(qa == QT_Q4_K && qb == QT_Q6_K) || K % 256 != 0 || B < 1 || B > 8 * MAXNT || n_sm < 2) return pp;
  const int NT = B <= 8 ? 1 : (B <= 16 ? 2 : 4);
  const int64_t U = K / 256;
  const double ba = (double)((Na + 15) / 16) * U * tile_bytes(qa), bb = (double)((Nb + 15) / 16) * U * tile_bytes(qb);
  pp.nA = std::min(n_sm - 1, std::max(1, (int)std::lround(n_sm * ba / (ba + bb))));
  for (int nt = NT; nt >= 1; nt >>= 1) {
    pp.a = make_plan(qa, Na, K, nt, pp.nA, max_smem, 16, 3, 0);
    pp.b = make_plan(qb, Nb, K, nt, n_sm - pp.nA, max_smem, 16, 3, 0);
    if (pp.a.NT == nt && pp.b.NT == nt) break;
  }
  if (pp.a.NT != pp.b.NT) return pp;
  const int nt = pp.a.NT;
  pp.partA = pp.a.geo.S > 1 ? (int64_t)pp.a.geo.S * pp.a.geo.T * 128 * nt : 0;
  pp.cntA = pp.a.geo.S > 1 ? pp.a.geo.T : 0;
  pp.partB = pp.b.geo.S > 1 ? (int64_t)pp.b.geo.S * pp.b.geo.T * 128 * nt : 0;
  pp.cntB = pp.b.geo.S > 1 ? pp.b.geo.T : 0;
  pp.ok = true;
  return pp;
}

void dev_limits(int device, int& n_sm, int& max_smem) {
  FAK_CUDA_CHECK(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device));
  FAK_CUDA_CHECK(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
}
}  // namespace

// Whether two matrices over the same activations can run as one pair launch, and the split-K
// scratch it needs: [] when not, else [CTAs of the first, floats, tickets].
std::vector<int64_t> tgemv_pair_plan(int64_t qa, int64_t Na, int64_t qb, int64_t Nb, int64_t K, int64_t B,
                                     int64_t device) {
  int n_sm = 0, max_smem = 0;
  dev_limits((int)device, n_sm, max_smem);
  const PairPlan pp = make_pair_plan((int)qa, Na, (int)qb, Nb, K, B, n_sm, max_smem);
  if (!pp.ok) return {};
  return {pp.nA, pp.partA + pp.partB, pp.cntA + pp.cntB};
}

// ya[:B] = Wa . x (+ bias_a) and yb[:B] = Wb . x (+ bias_b), EPI_STORE, in one launch per chunk of
// tokens; x quantized (qx, ds).  part / cnt hold both matrices' split-K scratch, the second's after
// the first's.
void tgemv_pair(torch::Tensor wa, int64_t qa, int64_t Na, torch::Tensor ya, c10::optional<torch::Tensor> bias_a,
                torch::Tensor wb, int64_t qb, int64_t Nb, torch::Tensor yb, c10::optional<torch::Tensor> bias_b,
                int64_t K, torch::Tensor qx, torch::Tensor ds, int64_t B, torch::Tensor part, torch::Tensor cnt,
                c10::optional<torch::Tensor> err, c10::optional<torch::Tensor> prefetch, bool unit) {
  static int n_sm = 0, max_smem = 0;
  if (!n_sm) dev_limits(wa.get_device(), n_sm, max_smem);
  const PairPlan pp = make_pair_plan((int)qa, Na, (int)qb, Nb, K, B, n_sm, max_smem);
  TORCH_CHECK(pp.ok, "tgemv_pair: no pair launch for these shapes (check tgemv_pair_plan first)");
  auto check_w = [&](const torch::Tensor& w, int64_t qt, int64_t N) {
    TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kUInt8 && reinterpret_cast<uintptr_t>(w.data_ptr()) % 16 == 0,
                "tgemv_pair: weights cuda uint8, 16-byte aligned");
    TORCH_CHECK(w.numel() >= (N + 15) / 16 * (K / 256) * tile_bytes((int)qt), "tgemv_pair: weight buffer too small");
  };
  check_w(wa, qa, Na);
  check_w(wb, qb, Nb);
  auto check_y = [&](const torch::Tensor& y, int64_t N, const c10::optional<torch::Tensor>& bias) -> const float* {
    TORCH_CHECK(y.scalar_type() == torch::kFloat32 && y.dim() == 2 && y.stride(1) == 1 && y.size(0) >= B &&
                    y.size(1) >= N, "tgemv_pair: y [B, >=N] f32");
    if (!bias.has_value()) return nullptr;
    TORCH_CHECK(bias->scalar_type() == torch::kFloat32 && bias->numel() >= N, "tgemv_pair: bias");
    return bias->data_ptr<float>();
  };
  const float* bpa = check_y(ya, Na, bias_a);
  const float* bpb = check_y(yb, Nb, bias_b);
  TORCH_CHECK(qx.scalar_type() == torch::kInt8 && qx.is_contiguous() && qx.numel() >= B * K &&
                  reinterpret_cast<uintptr_t>(qx.data_ptr()) % 16 == 0, "tgemv_pair: qx");
  TORCH_CHECK(ds.scalar_type() == torch::kFloat32 && ds.is_contiguous() && ds.numel() >= B * K / 16 &&
                  reinterpret_cast<uintptr_t>(ds.data_ptr()) % 16 == 0, "tgemv_pair: ds");
  TORCH_CHECK(part.scalar_type() == torch::kFloat32 && part.numel() >= pp.partA + pp.partB &&
                  cnt.scalar_type() == torch::kInt32 && cnt.numel() >= pp.cntA + pp.cntB, "tgemv_pair: scratch too small");
  auto args = [&](const torch::Tensor& w, int64_t N, const torch::Tensor& y, const float* bp, const Plan& p,
                  int64_t part_off, int64_t cnt_off) {
    TgArgs a{};
    a.Wt = w.data_ptr<uint8_t>();
    a.N = (int)N;
    a.K = (int)K;
    a.qx = qx.data_ptr<int8_t>();
    a.ds = reinterpret_cast<const float2*>(ds.data_ptr<float>());
    a.y = y.data_ptr<float>();
    a.ldy = y.stride(0);
    a.bias = bp;
    a.epi = EPI_STORE;
    a.part = p.geo.S > 1 ? part.data_ptr<float>() + part_off : nullptr;
    a.cnt = p.geo.S > 1 ? cnt.data_ptr<int>() + cnt_off : nullptr;
    a.err = err.has_value() ? err->data_ptr<int>() : nullptr;
    a.geo = p.geo;
    return a;
  };
  TgArgs A = args(wa, Na, ya, bpa, pp.a, 0, 0);
  TgArgs Bv = args(wb, Nb, yb, bpb, pp.b, pp.partA, pp.cntA);
  if (prefetch.has_value()) {
    A.pf = reinterpret_cast<const uint8_t*>(prefetch->data_ptr());
    A.pf_bytes = prefetch->numel() * prefetch->element_size();
  }
  const int nA = pp.a.geo.P * pp.a.geo.S, nB = pp.b.geo.P * pp.b.geo.S;
  const int smem = std::max(pp.a.smem, pp.b.smem);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(16 * 32);
  cfg.gridDim = dim3(nA + nB);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const int chunk = 8 * pp.a.NT;
  auto go = [&](auto kern) {
    FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    for (int64_t b0 = 0; b0 < B; b0 += chunk) {
      TgArgs a = A, b = Bv;
      a.B = b.B = (int)std::min<int64_t>(chunk, B - b0);
      a.qx = b.qx = A.qx + b0 * K;
      a.ds = b.ds = A.ds + b0 * (K / 32);
      a.y += b0 * a.ldy;
      b.y += b0 * b.ldy;
      if (b0 > 0) a.pf = nullptr;
      FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, a, b, nA));
    }
  };
#define FAK_TGP(NTV)                                                \
  {                                                                 \
    if (unit) go(k_tgemv_pair<QT_Q4_K, QT_Q6_K, 16, 3, NTV, true>); \
    else go(k_tgemv_pair<QT_Q4_K, QT_Q6_K, 16, 3, NTV, false>);     \
  }
  if (pp.a.NT == 1) FAK_TGP(1)
  else if (pp.a.NT == 2) FAK_TGP(2)
  else FAK_TGP(4)
#undef FAK_TGP
}

// Grouped expert GEMV over tile-packed experts (MoE decode).  w: tile-packed [E_local * rows_per_expert
// rows, K]; pairs grouped by moe_group (chunk_expert [max_chunks], chunk_pairs [max_chunks, 8], n_chunks [1]).
void moe_tgemv(torch::Tensor w, int64_t qtype, int64_t rows_per_expert, int64_t K, torch::Tensor qx,
               torch::Tensor ds, int64_t topk, bool act_by_token, torch::Tensor chunk_expert, torch::Tensor chunk_pairs,
               torch::Tensor n_chunks, int64_t max_chunks, torch::Tensor y, int64_t epi, torch::Tensor err,
               c10::optional<torch::Tensor> bias) {
  const float* bp = nullptr;
  if (bias.has_value()) {
    // the packed experts hold (bytes / bytes per expert) experts; the bias has rows_per_expert per expert
    const int64_t per_expert = (int64_t)tile_bytes((int)qtype) * (K / 256) * (rows_per_expert / 16);
    const int64_t n_exp = per_expert > 0 ? w.numel() / per_expert : 0;
    TORCH_CHECK(bias->is_cuda() && bias->scalar_type() == torch::kFloat32 && bias->is_contiguous() &&
                    bias->numel() >= n_exp * rows_per_expert, "moe_tgemv: bias [experts x rows per expert] f32");
    bp = bias->data_ptr<float>();
  }
  TORCH_CHECK(w.is_cuda() && w.scalar_type() == torch::kUInt8, "moe_tgemv: w");
  TORCH_CHECK(qtype == QT_Q4_K || qtype == QT_Q6_K || qtype == QT_Q8_0 || qtype == QT_G4, "moe_tgemv: qtype");
  TORCH_CHECK(rows_per_expert % 16 == 0 && K % 256 == 0, "moe_tgemv: rows per expert % 16, K % 256");
  TORCH_CHECK(qx.scalar_type() == torch::kInt8 && qx.is_contiguous() &&
                  reinterpret_cast<uintptr_t>(qx.data_ptr()) % 16 == 0, "moe_tgemv: qx");
  TORCH_CHECK(ds.scalar_type() == torch::kFloat32 && ds.is_contiguous() &&
                  reinterpret_cast<uintptr_t>(ds.data_ptr()) % 16 == 0, "moe_tgemv: ds");
  TORCH_CHECK(y.scalar_type() == torch::kFloat32 && y.stride(1) == 1, "moe_tgemv: y");
  TORCH_CHECK(chunk_pairs.numel() >= max_chunks * 8 && chunk_expert.numel() >= max_chunks, "moe_tgemv: chunks");
  static int max_smem = 0;
  if (!max_smem)
    FAK_CUDA_CHECK(cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, w.get_device()));
  TGeo g = make_geo((int)qtype, (int)(rows_per_expert / 16), (int)(K / 256), 1, 1);
  const int Te = (int)(rows_per_expert / 16);
  int W = 16, R = 3;
  if (tsmem((int)qtype, 16, 3, 1, g).total > max_smem) W = 8;
  TORCH_CHECK(tsmem((int)qtype, W, R, 1, g).total <= max_smem, "moe_tgemv: K too large for shared memory");
  const int smem = tsmem((int)qtype, W, R, 1, g).total;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(W * 32);
  cfg.gridDim = dim3((unsigned)max_chunks);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  auto go = [&](auto kern) {
    FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, (const uint8_t*)w.data_ptr<uint8_t>(), Te, (int)K,
                                      (const int8_t*)qx.data_ptr<int8_t>(),
                                      reinterpret_cast<const float2*>(ds.data_ptr<float>()), (int)topk,
                                      (int)act_by_token, (const int*)chunk_expert.data_ptr<int>(),
                                      (const int*)chunk_pairs.data_ptr<int>(), (const int*)n_chunks.data_ptr<int>(),
                                      y.data_ptr<float>(), (int64_t)y.stride(0), (int)epi, err.data_ptr<int>(), g, bp));
  };
#define FAK_TGM(QTV)                                       \
  {                                                        \
    if (W == 16) go(k_tgemv_moe<QTV, 16, 3>);              \
    else go(k_tgemv_moe<QTV, 8, 3>);                       \
  }
  if (qtype == QT_Q4_K) FAK_TGM(QT_Q4_K)
  else if (qtype == QT_G4) FAK_TGM(QT_G4)
  else if (qtype == QT_Q6_K) FAK_TGM(QT_Q6_K)
  else FAK_TGM(QT_Q8_0)
#undef FAK_TGM
}
