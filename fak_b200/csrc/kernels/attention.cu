// Paged attention over the block KV cache.
//
// KV layout: k_cache / v_cache [num_pages, Hkv, PAGE=16, D] bf16 -- one (page, kv-head) is one
// contiguous 16 x D tile, so a page streams with 16-byte async copies and its rows feed ldmatrix.
// Pages are shared between sequences through the radix prefix cache, so every sequence reads
// through its own block table.
//
// decode  (one query token per sequence): the query heads of one KV group are packed into the
//         M=16 rows of an m16n8k16 MMA (GQA groups <= 16), 16 tokens of one page are the N side;
//         the context is split across CTAs (flash-decode) and across the 4 warps of a CTA, with
//         an online softmax per warp and a log-sum-exp merge at the end.  The final merge writes
//         the output already quantized (int8 + per-32 scale/sum) for the o_proj GEMV.
//         Reference: k_flash_attention (internal/compute/cuda_kernels.cu:701-759), one block per
//         head over a contiguous f32 cache.
// prefill (a chunk of new tokens per sequence, after their K/V were appended): FlashAttention-2
//         style, 64 queries x one head per CTA, 64-token K/V tiles double-buffered in shared
//         memory, causal mask against absolute positions so a chunk attends to the whole cached
//         prefix plus itself.
#include <torch/extension.h>
#include <c10/cuda/CUDAStream.h>

#include <cstdio>
#include <cstdlib>
#include <mutex>

#include "mma.cuh"
#include "fak_noalloc.h"

using namespace fak;

namespace {

constexpr int PAGE = 16;
constexpr float NEG_INF = -INFINITY;

FAK_DEV float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
  return v;
}
FAK_DEV float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  v += __shfl_xor_sync(0xffffffffu, v, 2);
  return v;
}

// attention logit in the log2 domain: raw * scale * log2(e), or with soft-capping (cap_out > 0)
// cap * tanh(raw * scale / cap) * log2(e)  (cap_in = scale / cap, cap_out = cap * log2(e))
FAK_DEV float attn_logit(float raw, float scale_log2, float cap_in, float cap_out) {
  return cap_out > 0.f ? cap_out * tanhf(raw * cap_in) : raw * scale_log2;
}

// quantize one 32-wide block held one value per lane; writes int8 codes and (scale, sum of the
// dequantized values d * sum(codes))
FAK_DEV void warp_quant_store(float v, int8_t* qdst, float2* dsdst, int lane) {
  float amax = warp_max(fabsf(v));
  float d = amax / 127.f;
  const float q = d > 0.f ? rintf(v / d) : 0.f;
  const float s = warp_sum(q) * d;
  qdst[lane] = (int8_t)q;
  if (lane == 0) *dsdst = make_float2(d, s);
}

// =============================================================================================
// decode
// =============================================================================================
// Suffix splits of k_decode_attn that hold pages for a sequence of ctx tokens: the same page range
// arithmetic as the kernel (window start, pages another kernel covers, pages per split).
FAK_DEV int dec_live_splits(int ctx, int win, const int* skip_pages, int n_split, int pages_per_split) {
  const int n_pages = (ctx + PAGE - 1) / PAGE;
  int lo = win > 0 ? max(0, ctx - win) : 0;
  if (skip_pages != nullptr) lo = max(lo, min(ctx, *skip_pages * PAGE));
  const int live = n_pages - lo / PAGE;
  if (live <= 0) return 0;
  const int pps = max(pages_per_split, (live + n_split - 1) / n_split);
  return min(n_split, (live + pps - 1) / pps);
}

constexpr int kCombineMaxSlots = 384;   // 256 suffix splits + 128 cascade prefix splits

// Merge of one (sequence, head)'s split partials (o_s unnormalised, (m_s, l_s) in log2 units) by a
// 128-thread CTA: block max of the m_s, weights f_s = 2^(m_s - max) and L = sum f_s l_s, then each
// warp accumulates the splits s = warp (mod 4) with D/32 dims per lane and the four warps' sums
// are added in warp order.  Used by k_decode_combine and by the in-kernel merge (tickets), which
// therefore give the same bits.  Output: fp32 out and/or int8 codes with (scale, sum) per 32.
// sink2: the head's attention-sink logit in log2 units (-inf: none).
// smem: sf [kCombineMaxSlots], red [4 * D], s_red [8] floats.
template <int D>
FAK_DEV void combine_head(const float* __restrict__ part_o, const float2* __restrict__ part_ml, int64_t base,
                          int n_used, float* __restrict__ out, int8_t* __restrict__ qx, float2* __restrict__ ds,
                          int64_t oi0, float* sf, float* red, float* s_red, float sink2) {
  constexpr int VEC = D / 32;   // dims per lane
  constexpr int GL = 32 / VEC;  // lanes per 32-element quantization block
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  float mloc = NEG_INF;
  for (int s = tid; s < n_used; s += 128) mloc = fmaxf(mloc, __ldcg(&part_ml[base + s].x));
  mloc = warp_max(mloc);
  if (lane == 0) s_red[warp] = mloc;
  __syncthreads();
  // an attention sink (sink2 > -inf, log2 units) is one more logit of the softmax with no value
  const float mstar = fmaxf(fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3])), sink2);
  const float mb = mstar == NEG_INF ? 0.f : mstar;
  float lloc = 0.f;
  for (int s = tid; s < n_used; s += 128) {
    const float2 ml = __ldcg(&part_ml[base + s]);
    const float f = exp2f(ml.x - mb);
    sf[s] = f;
    lloc += f * ml.y;
  }
  lloc = warp_sum(lloc);
  if (lane == 0) s_red[4 + warp] = lloc;
  __syncthreads();
  const float L = (s_red[4] + s_red[5]) + (s_red[6] + s_red[7]) + (sink2 > NEG_INF ? exp2f(sink2 - mb) : 0.f);
  float acc[VEC];
#pragma unroll
  for (int e = 0; e < VEC; e++) acc[e] = 0.f;
  for (int s = warp; s < n_used; s += 4) {
    const float f = sf[s];
    const float* po = part_o + (base + s) * D + VEC * lane;
    if constexpr (VEC == 4) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(po));
      acc[0] += f * v.x; acc[1] += f * v.y; acc[2] += f * v.z; acc[3] += f * v.w;
    } else {
      const float2 v = __ldcg(reinterpret_cast<const float2*>(po));
      acc[0] += f * v.x; acc[1] += f * v.y;
    }
  }
#pragma unroll
  for (int e = 0; e < VEC; e++) red[(warp * 32 + lane) * VEC + e] = acc[e];
  __syncthreads();
  if (warp == 0) {
    float v[VEC];
#pragma unroll
    for (int e = 0; e < VEC; e++) {
      const float t = ((red[lane * VEC + e] + red[(32 + lane) * VEC + e]) + red[(64 + lane) * VEC + e]) +
                      red[(96 + lane) * VEC + e];
      v[e] = L > 0.f ? t / L : 0.f;
    }
    const int64_t oi = oi0 + VEC * lane;
    if (out) {
      if constexpr (VEC == 4) *reinterpret_cast<float4*>(out + oi) = make_float4(v[0], v[1], v[2], v[3]);
      else *reinterpret_cast<float2*>(out + oi) = make_float2(v[0], v[1]);
    }
    if (qx) {   // int8 per 32 elements with (scale, sum of the dequantized block), as warp_quant_store
      float amax = 0.f;
#pragma unroll
      for (int e = 0; e < VEC; e++) amax = fmaxf(amax, fabsf(v[e]));
#pragma unroll
      for (int o = GL / 2; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
      const float d = amax / 127.f;
      float qs = 0.f;
      uint32_t packed = 0;
#pragma unroll
      for (int e = 0; e < VEC; e++) {
        const float q = d > 0.f ? rintf(v[e] / d) : 0.f;
        qs += q;
        packed |= ((uint32_t)(int)q & 0xffu) << (8 * e);
      }
#pragma unroll
      for (int o = GL / 2; o; o >>= 1) qs += __shfl_xor_sync(0xffffffffu, qs, o);
      if constexpr (VEC == 4) *reinterpret_cast<uint32_t*>(qx + oi) = packed;
      else *reinterpret_cast<uint16_t*>(qx + oi) = (uint16_t)packed;
      if ((lane & (GL - 1)) == 0) ds[oi >> 5] = make_float2(d, qs * d);
    }
  }
  __syncthreads();   // sf / red / s_red are reused by the next head
}

// pages in flight per warp (ring depth).  Two pages (68 KB of shared memory at head dim 128) let
// three CTAs share an SM; three pages (102 KB) only two.  At 5 sequences x 4 KV heads x 16 splits
// (320 CTAs on 148 SMs) the deeper ring measured 28.0 us against 21.3 us for two.
constexpr int DEC_STAGES = 2;
template <int D, int ST = DEC_STAGES>
struct DecodeSmem {
  __nv_bfloat16 k[4][ST][PAGE][D + 8];
  __nv_bfloat16 v[4][ST][PAGE][D + 8];
};

template <int D, int ST = DEC_STAGES>   // ST: pages in flight per warp
__global__ void __launch_bounds__(128)
k_decode_attn(const float* __restrict__ q, const __nv_bfloat16* __restrict__ kc, const __nv_bfloat16* __restrict__ vc,
              const int* __restrict__ block_table, int bt_stride, const int* __restrict__ ctx_len, int H, int Hkv,
              int n_split, int pages_per_split, float scale_log2, float* __restrict__ part_o,
              float2* __restrict__ part_ml, float* __restrict__ out, int8_t* __restrict__ qx,
              float2* __restrict__ ds, int ldo, int* __restrict__ tickets, const uint8_t* __restrict__ pf,
              int64_t pf_bytes, int win, const int* __restrict__ skip_pages, int slot0, int n_slots, float cap_in,
              float cap_out, const float* __restrict__ sinks) {
  constexpr int KS = D / 16;   // k-steps over the head dim
  constexpr int NT = D / 8;    // n-tiles over the head dim for P.V
  extern __shared__ __align__(16) uint8_t smem_raw[];
  DecodeSmem<D, ST>& sm = *reinterpret_cast<DecodeSmem<D, ST>*>(smem_raw);

  const int kvh = blockIdx.x, b = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int G = H / Hkv;
  l2_prefetch(pf, pf_bytes);
  pdl_wait();
  const int ctx = ctx_len[b];
  const int n_pages = (ctx + PAGE - 1) / PAGE;
  // sliding window (win > 0): the query at ctx - 1 sees keys [ctx - win, ctx); pages before the
  // window are never read
  int lo = win > 0 ? max(0, ctx - win) : 0;
  if (skip_pages != nullptr) lo = max(lo, min(ctx, *skip_pages * PAGE));   // pages another kernel covers
  const int pg0 = lo / PAGE;
  // pages per split follow the live context so every split gets an even share of the pages
  const int pps = max(pages_per_split, (n_pages - pg0 + n_split - 1) / n_split);
  const int p_begin = pg0 + split * pps;
  const int p_end = min(n_pages, p_begin + pps);
  // a split past the live pages writes nothing: the combine reads only the live splits
  // (dec_live_splits); the in-kernel merge (tickets) needs every split's ticket, so it keeps them
  if (p_begin >= p_end && n_slots > 1 && tickets == nullptr) return;

  // Q fragments (rows = query heads of this group, zero beyond G)
  uint32_t qa[KS][4];
  {
    const int h0 = kvh * G + gq, h1 = kvh * G + gq + 8;
    const float* q0 = q + ((int64_t)b * H + h0) * D;
    const float* q1 = q + ((int64_t)b * H + h1) * D;
    const bool v0 = gq < G, v1 = gq + 8 < G;
#pragma unroll
    for (int ks = 0; ks < KS; ks++) {
      int c = ks * 16 + 2 * tq;
      float2 a0 = v0 ? *reinterpret_cast<const float2*>(q0 + c) : make_float2(0.f, 0.f);
      float2 a1 = v1 ? *reinterpret_cast<const float2*>(q1 + c) : make_float2(0.f, 0.f);
      float2 a2 = v0 ? *reinterpret_cast<const float2*>(q0 + c + 8) : make_float2(0.f, 0.f);
      float2 a3 = v1 ? *reinterpret_cast<const float2*>(q1 + c + 8) : make_float2(0.f, 0.f);
      qa[ks][0] = pack_bf16(a0.x, a0.y);
      qa[ks][1] = pack_bf16(a1.x, a1.y);
      qa[ks][2] = pack_bf16(a2.x, a2.y);
      qa[ks][3] = pack_bf16(a3.x, a3.y);
    }
  }
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = NEG_INF, m1 = NEG_INF, l0 = 0.f, l1 = 0.f;

  const int* bt = block_table + (int64_t)b * bt_stride;
  auto issue_page = [&](int p, int buf) {
    const int pid = bt[p];
    const __nv_bfloat16* ks = kc + ((int64_t)pid * Hkv + kvh) * PAGE * D;
    const __nv_bfloat16* vs = vc + ((int64_t)pid * Hkv + kvh) * PAGE * D;
    constexpr int CHUNKS = PAGE * D / 8;  // 16-byte chunks per tile
#pragma unroll
    for (int c = lane; c < CHUNKS; c += 32) {
      int tok = c / (D / 8), part = c % (D / 8);
      cp_async16(smem_u32(&sm.k[warp][buf][tok][part * 8]), ks + tok * D + part * 8);
      cp_async16(smem_u32(&sm.v[warp][buf][tok][part * 8]), vs + tok * D + part * 8);
    }
    cp_async_commit();
  };

  // warp w takes pages p_begin + w, + 4, ...; ST - 1 of them stay in flight while it
  // computes on one (an empty commit group keeps the group count uniform past the end)
  const int p0 = p_begin + warp;
#pragma unroll
  for (int i = 0; i < ST - 1; i++) {
    if (p0 + 4 * i < p_end) issue_page(p0 + 4 * i, i);
    else cp_async_commit();
  }
  int buf = 0;
  for (int p = p0, it = 0; p < p_end; p += 4, it++) {
    const int pn = p + 4 * (ST - 1);
    if (pn < p_end) issue_page(pn, (it + ST - 1) % ST);
    else cp_async_commit();
    cp_async_wait<ST - 1>();
    buf = it % ST;
    __syncwarp();
    // S = Q K^T for 16 tokens
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int jj = mi >> 1, hh = mi & 1;
#pragma unroll
      for (int ks = 0; ks < KS; ks++) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4(smem_u32(&sm.k[warp][buf][8 * jj + ri][16 * ks + 8 * hh]), r0, r1, r2, r3);
        mma_bf16_16816(s[0], qa[ks], r0, r1);
        mma_bf16_16816(s[1], qa[ks], r2, r3);
      }
    }
    const int valid = min(PAGE, ctx - p * PAGE), first = lo - p * PAGE;
#pragma unroll
    for (int j = 0; j < 2; j++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        int tok = 8 * j + 2 * tq + (e & 1);
        s[j][e] = (tok < valid && tok >= first) ? attn_logit(s[j][e], scale_log2, cap_in, cap_out) : NEG_INF;
      }
    }
    float mx0 = quad_max(fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1])));
    float mx1 = quad_max(fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3])));
    float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    float base0 = mn0 == NEG_INF ? 0.f : mn0, base1 = mn1 == NEG_INF ? 0.f : mn1;
    float c0 = exp2f(m0 - base0), c1 = exp2f(m1 - base1);
    m0 = mn0; m1 = mn1;
    float pr[2][4];
#pragma unroll
    for (int j = 0; j < 2; j++) {
      pr[j][0] = exp2f(s[j][0] - base0);
      pr[j][1] = exp2f(s[j][1] - base0);
      pr[j][2] = exp2f(s[j][2] - base1);
      pr[j][3] = exp2f(s[j][3] - base1);
    }
    l0 = l0 * c0 + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    l1 = l1 * c1 + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
#pragma unroll
    for (int i = 0; i < NT; i++) {
      o[i][0] *= c0; o[i][1] *= c0; o[i][2] *= c1; o[i][3] *= c1;
    }
    uint32_t pa[4] = {pack_bf16(pr[0][0], pr[0][1]), pack_bf16(pr[0][2], pr[0][3]), pack_bf16(pr[1][0], pr[1][1]),
                      pack_bf16(pr[1][2], pr[1][3])};
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int tok = (mi & 1) * 8 + ri, dsel = (mi >> 1) * 8;
#pragma unroll
      for (int d = 0; d < NT; d += 2) {
        uint32_t r0, r1, r2, r3;
        ldmatrix_x4_trans(smem_u32(&sm.v[warp][buf][tok][8 * d + dsel]), r0, r1, r2, r3);
        mma_bf16_16816(o[d], pa, r0, r1);
        mma_bf16_16816(o[d + 1], pa, r2, r3);
      }
    }
    __syncwarp();
  }
  cp_async_wait<0>();
  l0 = quad_sum(l0);
  l1 = quad_sum(l1);

  // merge the 4 warps through shared memory (reuses the K/V staging area)
  __syncthreads();
  float* so = reinterpret_cast<float*>(smem_raw);   // [4][16][D]
  float* sml = so + 4 * 16 * D;                      // [4][16][2]
#pragma unroll
  for (int i = 0; i < NT; i++) {
    int c = 8 * i + 2 * tq;
    so[(warp * 16 + gq) * D + c] = o[i][0];
    so[(warp * 16 + gq) * D + c + 1] = o[i][1];
    so[(warp * 16 + gq + 8) * D + c] = o[i][2];
    so[(warp * 16 + gq + 8) * D + c + 1] = o[i][3];
  }
  if (tq == 0) {
    sml[(warp * 16 + gq) * 2] = m0;
    sml[(warp * 16 + gq) * 2 + 1] = l0;
    sml[(warp * 16 + gq + 8) * 2] = m1;
    sml[(warp * 16 + gq + 8) * 2 + 1] = l1;
  }
  __syncthreads();
  pdl_launch_dependents();
  // each warp finalizes dims [32*warp, 32*warp+32) (D=128) or warps 0-1 (D=64) for every head
  for (int r = 0; r < G; r++) {
    const int h = kvh * G + r;
    // the attention sink joins the final softmax only (split partials leave it to the combine)
    const float sk = (n_slots == 1 && sinks != nullptr) ? sinks[h] * 1.4426950408889634f : NEG_INF;
    float mstar = NEG_INF;
#pragma unroll
    for (int w = 0; w < 4; w++) mstar = fmaxf(mstar, sml[(w * 16 + r) * 2]);
    const float mtot = fmaxf(mstar, sk);
    float base = mtot == NEG_INF ? 0.f : mtot;
    float L = sk > NEG_INF ? exp2f(sk - base) : 0.f, f[4];
#pragma unroll
    for (int w = 0; w < 4; w++) {
      f[w] = exp2f(sml[(w * 16 + r) * 2] - base);
      L += f[w] * sml[(w * 16 + r) * 2 + 1];
    }
    for (int dd = threadIdx.x; dd < D; dd += 128) {
      float acc = 0.f;
#pragma unroll
      for (int w = 0; w < 4; w++) acc += f[w] * so[(w * 16 + r) * D + dd];
      if (n_slots == 1) {
        float v = L > 0.f ? acc / L : 0.f;
        int64_t oi = (int64_t)b * ldo + (int64_t)h * D + dd;
        if (out) out[oi] = v;
        if (qx) warp_quant_store(v, qx + (oi & ~int64_t(31)), ds + (oi >> 5), lane);
      } else {
        int64_t pi = (((int64_t)b * H + h) * n_slots + slot0 + split);
        part_o[pi * D + dd] = acc;
        if (dd == 0) part_ml[pi] = make_float2(mstar, L);
      }
    }
  }
  if (n_slots == 1 || tickets == nullptr) return;   // (tickets are only passed with n_slots == n_split)
  // the last split CTA of this (sequence, KV group) merges all splits (same order and arithmetic
  // as k_decode_combine) and leaves its ticket at zero for the next launch
  __shared__ int s_ticket;
  __syncthreads();   // every thread's partial, then one fence ahead of the ticket
  if (threadIdx.x == 0) {
    __threadfence();
    s_ticket = atomicAdd(&tickets[b * Hkv + kvh], 1);
  }
  __syncthreads();
  if (s_ticket != n_split - 1) return;
  __threadfence();
  {
    // the page ring is drained: its shared memory holds the merge scratch
    float* sf = reinterpret_cast<float*>(smem_raw);
    float* red = sf + kCombineMaxSlots;
    float* s_red = red + 4 * D;
    const int n_used = dec_live_splits(ctx, win, skip_pages, n_split, pages_per_split);
    for (int r = 0; r < G; r++) {
      const int h = kvh * G + r;
      combine_head<D>(part_o, part_ml, ((int64_t)b * H + h) * n_split, n_used, out, qx, ds,
                      (int64_t)b * ldo + (int64_t)h * D, sf, red, s_red,
                      sinks != nullptr ? sinks[h] * 1.4426950408889634f : NEG_INF);
    }
  }
  if (threadIdx.x == 0) tickets[b * Hkv + kvh] = 0;
}

// ---------------------------------------------------------------------------------------------
// Shared-prefix ("cascade") decode attention: the first *shared_pages pages of every sequence's
// block table are the same physical pages (a radix-shared prompt prefix), so one CTA per (KV head,
// page range) streams each shared page into shared memory ONCE and attends it with the queries of
// every sequence in the batch: row r of the B*G query rows (sequence r / G, head kvh*G + r % G)
// belongs to warp r / 16.  Each warp writes its rows' unnormalised partials (o, max, sum) into
// slot `split` of the split-KV scratch; the per-sequence kernel covers the pages after the shared
// prefix in the remaining slots and k_decode_combine merges all of them.
// B*G <= 64 (four 16-row tiles).  Pages in flight per CTA: PREFIX_STAGES - 1.
constexpr int PREFIX_STAGES = 6;   // pages in flight per CTA: a CTA's whole page range is ~one round trip
template <int D>
struct PrefixSmem {
  __nv_bfloat16 k[PREFIX_STAGES][PAGE][D + 8];
  __nv_bfloat16 v[PREFIX_STAGES][PAGE][D + 8];
};

template <int D>
__global__ void __launch_bounds__(128)
k_decode_attn_prefix(const float* __restrict__ q, const __nv_bfloat16* __restrict__ kc,
                     const __nv_bfloat16* __restrict__ vc, const int* __restrict__ block_table, int bt_stride,
                     const int* __restrict__ shared_pages, int B, int H, int Hkv, int n_prefix_split,
                     float scale_log2, float* __restrict__ part_o, float2* __restrict__ part_ml, int n_slots,
                     float cap_in, float cap_out) {
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PrefixSmem<D>& sm = *reinterpret_cast<PrefixSmem<D>*>(smem_raw);
  const int kvh = blockIdx.x, split = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int G = H / Hkv, R = B * G;
  pdl_wait();
  const int n_shared = *shared_pages;
  const int pps = (n_shared + n_prefix_split - 1) / n_prefix_split;
  const int p_begin = min(n_shared, split * pps), p_end = min(n_shared, p_begin + pps);

  // this warp's 16 query rows
  const int r0 = warp * 16 + gq, r1 = r0 + 8;
  const bool v0 = r0 < R, v1 = r1 < R;
  const int b0 = r0 / G, h0 = kvh * G + r0 % G, b1 = r1 / G, h1 = kvh * G + r1 % G;
  uint32_t qa[KS][4];
  {
    const float* q0 = q + ((int64_t)b0 * H + h0) * D;
    const float* q1 = q + ((int64_t)b1 * H + h1) * D;
#pragma unroll
    for (int ks = 0; ks < KS; ks++) {
      int c = ks * 16 + 2 * tq;
      float2 a0 = v0 ? *reinterpret_cast<const float2*>(q0 + c) : make_float2(0.f, 0.f);
      float2 a1 = v1 ? *reinterpret_cast<const float2*>(q1 + c) : make_float2(0.f, 0.f);
      float2 a2 = v0 ? *reinterpret_cast<const float2*>(q0 + c + 8) : make_float2(0.f, 0.f);
      float2 a3 = v1 ? *reinterpret_cast<const float2*>(q1 + c + 8) : make_float2(0.f, 0.f);
      qa[ks][0] = pack_bf16(a0.x, a0.y);
      qa[ks][1] = pack_bf16(a1.x, a1.y);
      qa[ks][2] = pack_bf16(a2.x, a2.y);
      qa[ks][3] = pack_bf16(a3.x, a3.y);
    }
  }
  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = NEG_INF, m1 = NEG_INF, l0 = 0.f, l1 = 0.f;
  const bool active = warp * 16 < R;   // warps past the last row tile only help with the copies

  // the shared pages are identical in every block table: read them through sequence 0's row
  auto issue_page = [&](int p, int buf) {
    const int pid = block_table[p];
    const __nv_bfloat16* ks = kc + ((int64_t)pid * Hkv + kvh) * PAGE * D;
    const __nv_bfloat16* vs = vc + ((int64_t)pid * Hkv + kvh) * PAGE * D;
    constexpr int CHUNKS = PAGE * D / 8;
    for (int c = threadIdx.x; c < CHUNKS; c += 128) {
      int tok = c / (D / 8), part = c % (D / 8);
      cp_async16(smem_u32(&sm.k[buf][tok][part * 8]), ks + tok * D + part * 8);
      cp_async16(smem_u32(&sm.v[buf][tok][part * 8]), vs + tok * D + part * 8);
    }
    cp_async_commit();
  };
#pragma unroll
  for (int i = 0; i < PREFIX_STAGES - 1; i++) {
    if (p_begin + i < p_end) issue_page(p_begin + i, i);
    else cp_async_commit();
  }
  for (int p = p_begin, it = 0; p < p_end; p++, it++) {
    const int pn = p + PREFIX_STAGES - 1;
    // the slot refilled below was consumed in the previous iteration by every warp
    __syncthreads();
    if (pn < p_end) issue_page(pn, (it + PREFIX_STAGES - 1) % PREFIX_STAGES);
    else cp_async_commit();
    cp_async_wait<PREFIX_STAGES - 1>();
    __syncthreads();
    const int buf = it % PREFIX_STAGES;
    if (!active) continue;
    float s[2][4];
#pragma unroll
    for (int j = 0; j < 2; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int jj = mi >> 1, hh = mi & 1;
#pragma unroll
      for (int ks = 0; ks < KS; ks++) {
        uint32_t x0, x1, x2, x3;
        ldmatrix_x4(smem_u32(&sm.k[buf][8 * jj + ri][16 * ks + 8 * hh]), x0, x1, x2, x3);
        mma_bf16_16816(s[0], qa[ks], x0, x1);
        mma_bf16_16816(s[1], qa[ks], x2, x3);
      }
    }
#pragma unroll
    for (int j = 0; j < 2; j++)
#pragma unroll
      for (int e = 0; e < 4; e++) s[j][e] = attn_logit(s[j][e], scale_log2, cap_in, cap_out);   // full pages: no mask
    float mx0 = quad_max(fmaxf(fmaxf(s[0][0], s[0][1]), fmaxf(s[1][0], s[1][1])));
    float mx1 = quad_max(fmaxf(fmaxf(s[0][2], s[0][3]), fmaxf(s[1][2], s[1][3])));
    float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    float c0 = exp2f(m0 - mn0), c1 = exp2f(m1 - mn1);
    m0 = mn0;
    m1 = mn1;
    float pr[2][4];
#pragma unroll
    for (int j = 0; j < 2; j++) {
      pr[j][0] = exp2f(s[j][0] - mn0);
      pr[j][1] = exp2f(s[j][1] - mn0);
      pr[j][2] = exp2f(s[j][2] - mn1);
      pr[j][3] = exp2f(s[j][3] - mn1);
    }
    l0 = l0 * c0 + pr[0][0] + pr[0][1] + pr[1][0] + pr[1][1];
    l1 = l1 * c1 + pr[0][2] + pr[0][3] + pr[1][2] + pr[1][3];
#pragma unroll
    for (int i = 0; i < NT; i++) {
      o[i][0] *= c0; o[i][1] *= c0; o[i][2] *= c1; o[i][3] *= c1;
    }
    uint32_t pa[4] = {pack_bf16(pr[0][0], pr[0][1]), pack_bf16(pr[0][2], pr[0][3]), pack_bf16(pr[1][0], pr[1][1]),
                      pack_bf16(pr[1][2], pr[1][3])};
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int tok = (mi & 1) * 8 + ri, dsel = (mi >> 1) * 8;
#pragma unroll
      for (int d = 0; d < NT; d += 2) {
        uint32_t x0, x1, x2, x3;
        ldmatrix_x4_trans(smem_u32(&sm.v[buf][tok][8 * d + dsel]), x0, x1, x2, x3);
        mma_bf16_16816(o[d], pa, x0, x1);
        mma_bf16_16816(o[d + 1], pa, x2, x3);
      }
    }
  }
  cp_async_wait<0>();
  pdl_launch_dependents();
  if (!active) return;
  l0 = quad_sum(l0);
  l1 = quad_sum(l1);
  // partials of this warp's rows (an empty range leaves max -inf, sum 0)
  const int64_t pi0 = (((int64_t)b0 * H + h0) * n_slots + split), pi1 = (((int64_t)b1 * H + h1) * n_slots + split);
#pragma unroll
  for (int i = 0; i < NT; i++) {
    const int c = 8 * i + 2 * tq;
    if (v0) *reinterpret_cast<float2*>(part_o + pi0 * D + c) = make_float2(o[i][0], o[i][1]);
    if (v1) *reinterpret_cast<float2*>(part_o + pi1 * D + c) = make_float2(o[i][2], o[i][3]);
  }
  if (tq == 0) {
    if (v0) part_ml[pi0] = make_float2(m0, l0);
    if (v1) part_ml[pi1] = make_float2(m1, l1);
  }
}

// Merges slots [0, slot0) (cascade prefix splits, all written) and the live suffix splits
// [slot0, slot0 + live) of each (sequence, head); splits past a sequence's pages wrote nothing.
template <int D>
__global__ void __launch_bounds__(128)
k_decode_combine(const float* __restrict__ part_o, const float2* __restrict__ part_ml, int H, int n_slots,
                 float* __restrict__ out, int8_t* __restrict__ qx, float2* __restrict__ ds, int ldo,
                 const int* __restrict__ ctx_len, int win, const int* __restrict__ skip_pages, int slot0, int n_split,
                 int pages_per_split, const float* __restrict__ sinks) {
  __shared__ float sf[kCombineMaxSlots];
  __shared__ float red[4 * D];
  __shared__ float s_red[8];
  pdl_wait();
  const int b = blockIdx.x, h = blockIdx.y;
  const int64_t base = ((int64_t)b * H + h) * n_slots;
  const int n_used = slot0 + dec_live_splits(ctx_len[b], win, skip_pages, n_split, pages_per_split);
  combine_head<D>(part_o, part_ml, base, n_used, out, qx, ds, (int64_t)b * ldo + (int64_t)h * D, sf, red, s_red,
                  sinks != nullptr ? sinks[h] * 1.4426950408889634f : NEG_INF);
  pdl_launch_dependents();
}

// =============================================================================================
// prefill
// =============================================================================================
constexpr int PF_Q = 64;   // queries per CTA (4 warps x 16)
constexpr int PF_KV = 64;  // keys per tile

template <int D>
struct PrefillSmem {
  __nv_bfloat16 k[2][PF_KV][D + 8];
  __nv_bfloat16 v[2][PF_KV][D + 8];
};

// CAP: soft-capped logits; WIN: sliding-window mask.  Separate instantiations keep the plain
// causal kernel free of both (measured 8% slower when they were runtime options).
// The plain variant compiles to 168 registers at head dim 128 on its own (3 CTAs per SM); the
// capped / windowed ones are held to that with a launch bound (a bound on the plain one measured
// 6% slower).
template <int D, bool CAP, bool WIN>
__global__ void __launch_bounds__(128, (D == 128 && (CAP || WIN)) ? 3 : 0)
k_prefill_attn(const __nv_bfloat16* __restrict__ q, int64_t q_stride, const __nv_bfloat16* __restrict__ kc,
               const __nv_bfloat16* __restrict__ vc, const int* __restrict__ block_table, int bt_stride,
               const int* __restrict__ tile_seq, const int* __restrict__ tile_q0, const int* __restrict__ seq_qoff,
               const int* __restrict__ seq_qlen, const int* __restrict__ seq_pos0, int H, int Hkv, float scale_log2,
               __nv_bfloat16* __restrict__ out, int64_t out_stride, int win, float cap_in, float cap_out,
               const float* __restrict__ sinks) {
  constexpr int KS = D / 16;
  constexpr int NT = D / 8;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PrefillSmem<D>& sm = *reinterpret_cast<PrefillSmem<D>*>(smem_raw);
  const int tile = blockIdx.x, h = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int G = H / Hkv, kvh = h / G;
  pdl_wait();
  const int sq = tile_seq[tile];
  const int q0 = tile_q0[tile];
  const int qoff = seq_qoff[sq], qlen = seq_qlen[sq], pos0 = seq_pos0[sq];
  const int* bt = block_table + (int64_t)sq * bt_stride;

  const int r0 = q0 + warp * 16 + gq, r1 = r0 + 8;  // local query indices of this thread's rows
  const bool v0 = r0 < qlen, v1 = r1 < qlen;
  uint32_t qa[KS][4];
  {
    const __nv_bfloat16* qp0 = q + (int64_t)(qoff + r0) * q_stride + (int64_t)h * D;
    const __nv_bfloat16* qp1 = q + (int64_t)(qoff + r1) * q_stride + (int64_t)h * D;
#pragma unroll
    for (int ks = 0; ks < KS; ks++) {
      int c = ks * 16 + 2 * tq;
      qa[ks][0] = v0 ? *reinterpret_cast<const uint32_t*>(qp0 + c) : 0u;
      qa[ks][1] = v1 ? *reinterpret_cast<const uint32_t*>(qp1 + c) : 0u;
      qa[ks][2] = v0 ? *reinterpret_cast<const uint32_t*>(qp0 + c + 8) : 0u;
      qa[ks][3] = v1 ? *reinterpret_cast<const uint32_t*>(qp1 + c + 8) : 0u;
    }
  }
  const int qpos0 = pos0 + r0, qpos1 = pos0 + r1;
  // lowest visible key of each row minus one (sliding window), or below every position
  const int lo0 = WIN ? qpos0 - win : -1, lo1 = WIN ? qpos1 - win : -1;
  const int kv_end = pos0 + min(q0 + PF_Q, qlen);  // exclusive bound on keys any row of this tile sees
  const int n_kv_tiles = (kv_end + PF_KV - 1) / PF_KV;

  float o[NT][4];
#pragma unroll
  for (int i = 0; i < NT; i++) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = NEG_INF, m1 = NEG_INF, l0 = 0.f, l1 = 0.f;

  auto issue_tile = [&](int kt, int buf) {
    constexpr int CPR = D / 8;  // 16-byte chunks per token row
    for (int c = threadIdx.x; c < PF_KV * CPR; c += 128) {
      int tok = c / CPR, part = c % CPR;
      int kp = kt * PF_KV + tok;
      bool ok = kp < kv_end;
      int pid = ok ? bt[kp / PAGE] : 0;
      int64_t off = (((int64_t)pid * Hkv + kvh) * PAGE + (kp % PAGE)) * D + part * 8;
      cp_async16_zfill(smem_u32(&sm.k[buf][tok][part * 8]), kc + (ok ? off : 0), ok);
      cp_async16_zfill(smem_u32(&sm.v[buf][tok][part * 8]), vc + (ok ? off : 0), ok);
    }
    cp_async_commit();
  };

  // sliding window (win > 0): row qp sees keys (qp - win, qp]; key tiles below the first row's
  // window are skipped
  const int kt0 = WIN ? max(0, pos0 + q0 - win + 1) / PF_KV : 0;
  if (kt0 < n_kv_tiles) issue_tile(kt0, kt0 & 1);
  for (int kt = kt0; kt < n_kv_tiles; kt++) {
    const int buf = kt & 1;
    if (kt + 1 < n_kv_tiles) {
      issue_tile(kt + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; j++) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int jj = mi >> 1, hh = mi & 1;
#pragma unroll
      for (int ks = 0; ks < KS; ks++) {
#pragma unroll
        for (int jp = 0; jp < 4; jp++) {  // pairs of n-tiles (16 keys)
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(smem_u32(&sm.k[buf][16 * jp + 8 * jj + ri][16 * ks + 8 * hh]), b0, b1, b2, b3);
          mma_bf16_16816(s[2 * jp], qa[ks], b0, b1);
          mma_bf16_16816(s[2 * jp + 1], qa[ks], b2, b3);
        }
      }
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
#pragma unroll
      for (int e = 0; e < 4; e++) {
        int kp = kt * PF_KV + 8 * j + 2 * tq + (e & 1);
        int qp = (e < 2) ? qpos0 : qpos1;
        int lo = (e < 2) ? lo0 : lo1;
        const float lg = CAP ? cap_out * tanhf(s[j][e] * cap_in) : s[j][e] * scale_log2;
        s[j][e] = (kp <= qp && (!WIN || kp > lo) && kp < kv_end) ? lg : NEG_INF;
      }
    }
    float mx0 = NEG_INF, mx1 = NEG_INF;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = quad_max(mx0);
    mx1 = quad_max(mx1);
    float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    float base0 = mn0 == NEG_INF ? 0.f : mn0, base1 = mn1 == NEG_INF ? 0.f : mn1;
    float c0 = exp2f(m0 - base0), c1 = exp2f(m1 - base1);
    m0 = mn0; m1 = mn1;
    float rs0 = 0.f, rs1 = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      s[j][0] = exp2f(s[j][0] - base0);
      s[j][1] = exp2f(s[j][1] - base0);
      s[j][2] = exp2f(s[j][2] - base1);
      s[j][3] = exp2f(s[j][3] - base1);
      rs0 += s[j][0] + s[j][1];
      rs1 += s[j][2] + s[j][3];
    }
    l0 = l0 * c0 + rs0;
    l1 = l1 * c1 + rs1;
#pragma unroll
    for (int i = 0; i < NT; i++) {
      o[i][0] *= c0; o[i][1] *= c0; o[i][2] *= c1; o[i][3] *= c1;
    }
    {
      const int mi = lane >> 3, ri = lane & 7;
      const int tsel = (mi & 1) * 8 + ri, dsel = (mi >> 1) * 8;
#pragma unroll
      for (int kk = 0; kk < 4; kk++) {
        uint32_t pa[4] = {pack_bf16(s[2 * kk][0], s[2 * kk][1]), pack_bf16(s[2 * kk][2], s[2 * kk][3]),
                          pack_bf16(s[2 * kk + 1][0], s[2 * kk + 1][1]), pack_bf16(s[2 * kk + 1][2], s[2 * kk + 1][3])};
#pragma unroll
        for (int d = 0; d < NT; d += 2) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(smem_u32(&sm.v[buf][16 * kk + tsel][8 * d + dsel]), b0, b1, b2, b3);
          mma_bf16_16816(o[d], pa, b0, b1);
          mma_bf16_16816(o[d + 1], pa, b2, b3);
        }
      }
    }
    __syncthreads();
  }
  pdl_launch_dependents();
  l0 = quad_sum(l0);
  l1 = quad_sum(l1);
  if (sinks != nullptr) {   // the head's sink logit joins each row's softmax denominator
    const float sk = sinks[h] * 1.4426950408889634f;
    l0 += exp2f(sk - m0);
    l1 += exp2f(sk - m1);
  }
  float inv0 = l0 > 0.f ? 1.f / l0 : 0.f, inv1 = l1 > 0.f ? 1.f / l1 : 0.f;
  __nv_bfloat16* op0 = out + (int64_t)(qoff + r0) * out_stride + (int64_t)h * D;
  __nv_bfloat16* op1 = out + (int64_t)(qoff + r1) * out_stride + (int64_t)h * D;
#pragma unroll
  for (int i = 0; i < NT; i++) {
    int c = 8 * i + 2 * tq;
    if (v0) *reinterpret_cast<uint32_t*>(op0 + c) = pack_bf16(o[i][0] * inv0, o[i][1] * inv0);
    if (v1) *reinterpret_cast<uint32_t*>(op1 + c) = pack_bf16(o[i][2] * inv1, o[i][3] * inv1);
  }
}

cudaLaunchAttribute g_pdl_attr[1];

void set_pdl(cudaLaunchConfig_t& cfg) {
  g_pdl_attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  g_pdl_attr[0].val.programmaticStreamSerializationAllowed = fak::pdl_allowed();
  cfg.attrs = g_pdl_attr;
  cfg.numAttrs = 1;
}

}  // namespace

// q [B,H,D] f32; caches [P,Hkv,16,D] bf16; block_table [B, *] int32; ctx_len [B] int32.
// Writes out [B,H*D] f32 (optional) and/or the int8 quantized output (qx [B,H*D], ds [B,H*D/32,2]).
// workspace: f32 buffer of at least B*H*n_split*(D+2) floats when n_split > 1.
// window > 0: sliding-window attention (the last ``window`` keys of each sequence).
void decode_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                      torch::Tensor ctx_len, int64_t n_split, int64_t pages_per_split,
                      c10::optional<torch::Tensor> out, c10::optional<torch::Tensor> qx,
                      c10::optional<torch::Tensor> ds, c10::optional<torch::Tensor> workspace, int64_t ldo,
                      c10::optional<torch::Tensor> tickets, c10::optional<torch::Tensor> prefetch, int64_t window,
                      c10::optional<torch::Tensor> shared_pages, int64_t prefix_splits, double scale, double softcap,
                      c10::optional<torch::Tensor> sinks) {
  const float* skp = nullptr;   // attention sinks [H] f32 (natural-log logits), optional
  if (sinks.has_value()) {
    TORCH_CHECK(sinks->is_cuda() && sinks->scalar_type() == torch::kFloat32 && sinks->numel() >= q.size(1),
                "decode_attention: sinks [H] f32");
    skp = sinks->data_ptr<float>();
  }
  const uint8_t* pfp = prefetch.has_value() ? reinterpret_cast<const uint8_t*>(prefetch->data_ptr()) : nullptr;
  const int64_t pfb = prefetch.has_value() ? prefetch->numel() * prefetch->element_size() : 0;
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kFloat32 && q.dim() == 3 && q.is_contiguous(), "q [B,H,D] f32");
  TORCH_CHECK(k_cache.scalar_type() == torch::kBFloat16 && k_cache.dim() == 4 && k_cache.is_contiguous(), "k_cache");
  TORCH_CHECK(v_cache.sizes() == k_cache.sizes() && v_cache.is_contiguous(), "v_cache");
  TORCH_CHECK(k_cache.size(2) == PAGE, "page size must be 16");
  int B = (int)q.size(0), H = (int)q.size(1), D = (int)q.size(2), Hkv = (int)k_cache.size(1);
  TORCH_CHECK(k_cache.size(3) == D && (D == 64 || D == 128), "head dim must be 64 or 128");
  TORCH_CHECK(H % Hkv == 0 && H / Hkv <= 16, "GQA group must be <= 16");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && block_table.dim() == 2 && block_table.stride(1) == 1, "bt");
  TORCH_CHECK(ctx_len.scalar_type() == torch::kInt32 && ctx_len.numel() >= B, "ctx_len");
  TORCH_CHECK(n_split >= 1 && pages_per_split >= 1, "split");
  if (B == 0) return;
  float* op = out.has_value() ? out->data_ptr<float>() : nullptr;
  int8_t* qp = qx.has_value() ? qx->data_ptr<int8_t>() : nullptr;
  float2* dp = ds.has_value() ? reinterpret_cast<float2*>(ds->data_ptr<float>()) : nullptr;
  if (ldo <= 0) ldo = (int64_t)H * D;  // elements per token row of out / qx
  TORCH_CHECK(ldo >= (int64_t)H * D && ldo % 32 == 0, "decode_attention: output row stride");
  const int64_t need = (int64_t)(B - 1) * ldo + (int64_t)H * D;  // last element written + 1
  if (qp) TORCH_CHECK(dp && qx->numel() >= need && ds->numel() >= need / 16, "qx/ds size");
  if (op) TORCH_CHECK(out->numel() >= need && out->is_contiguous(), "out");
  // cascade: the first *shared_pages pages (the same physical pages in every block table) are
  // attended once for the whole batch by k_decode_attn_prefix in prefix_splits extra slots
  const bool cascade = shared_pages.has_value() && prefix_splits > 0 && B * (H / Hkv) <= 64 && window <= 0;
  const int64_t n_slots = n_split + (cascade ? prefix_splits : 0);
  TORCH_CHECK(n_slots <= kCombineMaxSlots, "decode_attention: at most ", kCombineMaxSlots, " split slots");
  if (cascade)
    TORCH_CHECK(shared_pages->is_cuda() && shared_pages->scalar_type() == torch::kInt32 && shared_pages->numel() >= 1,
                "decode_attention: shared_pages int32 [1] on the device");
  float* pw = nullptr;
  if (n_slots > 1) {
    TORCH_CHECK(workspace.has_value() && workspace->scalar_type() == torch::kFloat32 &&
                    workspace->numel() >= (int64_t)B * H * n_slots * (D + 2),
                "decode_attention: workspace too small");
    pw = workspace->data_ptr<float>();
  }
  float2* pml = pw ? reinterpret_cast<float2*>(pw + (int64_t)B * H * n_slots * D) : nullptr;
  int* tk = nullptr;  // given: the last split CTA merges (no combine launch)
  if (n_split > 1 && tickets.has_value() && !cascade) {
    TORCH_CHECK(tickets->scalar_type() == torch::kInt32 && tickets->numel() >= (int64_t)B * Hkv,
                "decode_attention: tickets [B * Hkv] int32");
    tk = tickets->data_ptr<int>();
  }
  // logit scale (default 1/sqrt(D)) and optional soft-cap, in the log2 domain of the kernels
  const float sc = scale > 0 ? (float)scale : 1.0f / sqrtf((float)D);
  float scale_log2 = sc * 1.4426950408889634f;
  const float cap_in = softcap > 0 ? sc / (float)softcap : 0.f;
  const float cap_out = softcap > 0 ? (float)softcap * 1.4426950408889634f : 0.f;
  auto stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(Hkv, B, (unsigned)n_split);
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  set_pdl(cfg);
  int bts = (int)block_table.stride(0);
  const int* skip = cascade ? shared_pages->data_ptr<int>() : nullptr;
  const int slot0 = cascade ? (int)prefix_splits : 0;
  if (cascade) {
    cudaLaunchConfig_t cp = {};
    cp.gridDim = dim3(Hkv, (unsigned)prefix_splits);
    cp.blockDim = dim3(128);
    cp.stream = stream;
    set_pdl(cp);
    auto go = [&](auto kern, size_t smem) {
      cp.dynamicSmemBytes = smem;
      FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
      FAK_CUDA_CHECK(cudaLaunchKernelEx(&cp, kern, (const float*)q.data_ptr<float>(),
                                        (const __nv_bfloat16*)k_cache.data_ptr(),
                                        (const __nv_bfloat16*)v_cache.data_ptr(),
                                        (const int*)block_table.data_ptr<int>(), bts, skip, B, H, Hkv,
                                        (int)prefix_splits, scale_log2, pw, pml, (int)n_slots, cap_in, cap_out));
    };
    if (D == 128) go(k_decode_attn_prefix<128>, sizeof(PrefixSmem<128>));
    else go(k_decode_attn_prefix<64>, sizeof(PrefixSmem<64>));
  }
  // page-ring depth per warp: DEC_STAGES (2), or 3 with FAK_DEC_STAGES=3
  static const int dec_st = [] {
    const char* e = std::getenv("FAK_DEC_STAGES");
    return (e && std::atoi(e) == 3) ? 3 : DEC_STAGES;
  }();
  auto go = [&](auto kern, size_t smem) {
    cfg.dynamicSmemBytes = smem;
    FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FAK_CUDA_CHECK(cudaLaunchKernelEx(&cfg, kern, (const float*)q.data_ptr<float>(),
                                      (const __nv_bfloat16*)k_cache.data_ptr(), (const __nv_bfloat16*)v_cache.data_ptr(),
                                      (const int*)block_table.data_ptr<int>(), bts, (const int*)ctx_len.data_ptr<int>(),
                                      H, Hkv, (int)n_split, (int)pages_per_split, scale_log2, pw, pml, op, qp, dp, (int)ldo, tk,
                                      pfp, pfb, (int)window, skip, slot0, (int)n_slots, cap_in, cap_out, skp));
  };
  const size_t merge128 = (size_t)(4 * 16 * 128 + 4 * 16 * 2) * 4, merge64 = (size_t)(4 * 16 * 64 + 4 * 16 * 2) * 4;
  if (D == 128) {
    if (dec_st == 2) go(k_decode_attn<128, 2>, std::max(sizeof(DecodeSmem<128, 2>), merge128));
    else go(k_decode_attn<128, 3>, std::max(sizeof(DecodeSmem<128, 3>), merge128));
  } else {
    if (dec_st == 2) go(k_decode_attn<64, 2>, std::max(sizeof(DecodeSmem<64, 2>), merge64));
    else go(k_decode_attn<64, 3>, std::max(sizeof(DecodeSmem<64, 3>), merge64));
  }
  if (n_slots > 1 && tk == nullptr) {
    cudaLaunchConfig_t c2 = {};
    c2.gridDim = dim3(B, H);
    c2.blockDim = dim3(128);
    c2.stream = stream;
    set_pdl(c2);
    const int* cl = (const int*)ctx_len.data_ptr<int>();
    if (D == 128)
      FAK_CUDA_CHECK(cudaLaunchKernelEx(&c2, k_decode_combine<128>, (const float*)pw, (const float2*)pml, H,
                                        (int)n_slots, op, qp, dp, (int)ldo, cl, (int)window, skip, slot0, (int)n_split,
                                        (int)pages_per_split, skp));
    else
      FAK_CUDA_CHECK(cudaLaunchKernelEx(&c2, k_decode_combine<64>, (const float*)pw, (const float2*)pml, H,
                                        (int)n_slots, op, qp, dp, (int)ldo, cl, (int)window, skip, slot0, (int)n_split,
                                        (int)pages_per_split, skp));
  }
}

// q [T,H,D] bf16 (row stride q_stride elements); out [T, H*D] bf16 (row stride out_stride).
// Per-tile metadata (int32, device): tile_seq, tile_q0; per-sequence: seq_qoff, seq_qlen, seq_pos0.
void prefill_attention(torch::Tensor q, torch::Tensor k_cache, torch::Tensor v_cache, torch::Tensor block_table,
                       torch::Tensor tile_seq, torch::Tensor tile_q0, torch::Tensor seq_qoff, torch::Tensor seq_qlen,
                       torch::Tensor seq_pos0, int64_t n_tiles, torch::Tensor out, int64_t window, double scale,
                       double softcap, c10::optional<torch::Tensor> sinks) {
  TORCH_CHECK(q.is_cuda() && q.scalar_type() == torch::kBFloat16 && q.dim() == 3 && q.stride(2) == 1, "q [T,H,D] bf16");
  const float* skp = nullptr;   // attention sinks [H] f32 (natural-log logits), optional
  if (sinks.has_value()) {
    TORCH_CHECK(sinks->is_cuda() && sinks->scalar_type() == torch::kFloat32 && sinks->numel() >= q.size(1),
                "prefill_attention: sinks [H] f32");
    skp = sinks->data_ptr<float>();
  }
  TORCH_CHECK(k_cache.scalar_type() == torch::kBFloat16 && k_cache.dim() == 4 && k_cache.is_contiguous(), "k_cache");
  int H = (int)q.size(1), D = (int)q.size(2), Hkv = (int)k_cache.size(1);
  TORCH_CHECK(q.stride(1) == D, "q heads must be contiguous");
  TORCH_CHECK(D == 64 || D == 128, "head dim must be 64 or 128");
  TORCH_CHECK(out.scalar_type() == torch::kBFloat16 && out.dim() == 2 && out.stride(1) == 1, "out [T,H*D] bf16");
  TORCH_CHECK(block_table.scalar_type() == torch::kInt32 && block_table.stride(1) == 1, "block_table");
  if (n_tiles == 0) return;
  // logit scale (default 1/sqrt(D)) and optional soft-cap, in the log2 domain of the kernels
  const float sc = scale > 0 ? (float)scale : 1.0f / sqrtf((float)D);
  float scale_log2 = sc * 1.4426950408889634f;
  const float cap_in = softcap > 0 ? sc / (float)softcap : 0.f;
  const float cap_out = softcap > 0 ? (float)softcap * 1.4426950408889634f : 0.f;
  auto stream = at::cuda::getCurrentCUDAStream();
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_tiles, H);
  cfg.blockDim = dim3(128);
  cfg.stream = stream;
  set_pdl(cfg);
  auto args = [&](auto kern, size_t smem) {
    cfg.dynamicSmemBytes = smem;
    FAK_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    FAK_CUDA_CHECK(cudaLaunchKernelEx(
        &cfg, kern, (const __nv_bfloat16*)q.data_ptr(), (int64_t)q.stride(0), (const __nv_bfloat16*)k_cache.data_ptr(),
        (const __nv_bfloat16*)v_cache.data_ptr(), (const int*)block_table.data_ptr<int>(), (int)block_table.stride(0),
        (const int*)tile_seq.data_ptr<int>(), (const int*)tile_q0.data_ptr<int>(), (const int*)seq_qoff.data_ptr<int>(),
        (const int*)seq_qlen.data_ptr<int>(), (const int*)seq_pos0.data_ptr<int>(), H, Hkv, scale_log2,
        (__nv_bfloat16*)out.data_ptr(), (int64_t)out.stride(0), (int)window, cap_in, cap_out, skp));
  };
  const bool cap = cap_out > 0.f, wn = window > 0;
#define FAK_PF(DV)                                                                              \
  {                                                                                             \
    if (cap && wn) args(k_prefill_attn<DV, true, true>, sizeof(PrefillSmem<DV>));               \
    else if (cap) args(k_prefill_attn<DV, true, false>, sizeof(PrefillSmem<DV>));               \
    else if (wn) args(k_prefill_attn<DV, false, true>, sizeof(PrefillSmem<DV>));                \
    else args(k_prefill_attn<DV, false, false>, sizeof(PrefillSmem<DV>));                       \
  }
  if (D == 128) FAK_PF(128)
  else FAK_PF(64)
#undef FAK_PF
}

// =============================================================================================
// fak_decode_attention_noalloc: the split-KV decode attention above, as one C entry point that
// allocates nothing.  This entry point has no counterpart in the reference.  Its declaration, the
// callers it serves (runtimes that cannot allocate device memory while they run), its limits, the
// set-up rule and the concurrency rule are in fak_noalloc.h beside this file; the definition
// below must keep that signature (the header is included above, so the compiler checks it).
// =============================================================================================
namespace {
constexpr int64_t kNoAllocSlots = FAK_NOALLOC_MAX_SLOTS;
constexpr int kNoAllocMaxD = 128;
constexpr int kNoAllocMaxDevices = 64;
__device__ __align__(256) float g_noalloc_scratch[kNoAllocSlots * (kNoAllocMaxD + 2)];
std::mutex g_noalloc_mu;
float* g_noalloc_ptr[kNoAllocMaxDevices] = {};
static_assert(sizeof(g_noalloc_scratch) == 2129920, "the scratch size stated in fak_noalloc.h");

template <typename... A>
int noalloc_fail(char* err, size_t err_len, int code, const char* fmt, A... a) {
  if (err && err_len) {
    if constexpr (sizeof...(A) == 0) snprintf(err, err_len, "%s", fmt);
    else snprintf(err, err_len, fmt, a...);
  }
  return code;
}
}  // namespace

extern "C" __attribute__((visibility("default"))) int fak_decode_attention_noalloc(
    const float* q, const void* k_cache, const void* v_cache, const int* block_table, int bt_stride,
    const int* ctx_len, int B, int H, int Hkv, int D, int n_split, int pages_per_split, float* out, int8_t* qx,
    float* ds, int ldo, void* stream, char* err, size_t err_len) {
  if (err && err_len) err[0] = 0;
  if (!q || !k_cache || !v_cache || !block_table || !ctx_len)
    return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: null input pointer");
  if (!out && !qx) return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: no output (out or qx)");
  if (qx && !ds) return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: qx given without ds");
  if (D != 64 && D != 128)
    return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: head dim %d (must be 64 or 128)", D);
  if (B < 0 || H <= 0 || Hkv <= 0 || H % Hkv != 0 || H / Hkv > 16)
    return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: heads %d / kv heads %d (GQA group <= 16)", H,
                        Hkv);
  if (n_split < 1 || pages_per_split < 1 || bt_stride < 1)
    return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: n_split, pages_per_split, bt_stride >= 1");
  if (ldo <= 0) ldo = H * D;
  if (ldo < H * D || ldo % 32 != 0)
    return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: output row stride %d", ldo);
  const int64_t slots = (int64_t)B * H * n_split;
  if (n_split > kCombineMaxSlots)
    return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: n_split %d above %d", n_split,
                        kCombineMaxSlots);
  if (n_split > 1 && slots > kNoAllocSlots)
    return noalloc_fail(err, err_len, FAK_NOALLOC_ETOOBIG,
                        "fak_decode_attention_noalloc: B*H*n_split = %lld exceeds the static scratch limit of %lld "
                        "slots (%lld bytes); use fewer splits or the allocating entry point",
                        (long long)slots, (long long)kNoAllocSlots,
                        (long long)(kNoAllocSlots * (kNoAllocMaxD + 2) * sizeof(float)));
  if (B == 0) return FAK_NOALLOC_OK;

  float* pw = nullptr;
  if (n_split > 1) {
    int dev = -1;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return noalloc_fail(err, err_len, FAK_NOALLOC_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kNoAllocMaxDevices)
      return noalloc_fail(err, err_len, FAK_NOALLOC_EINVAL, "fak_decode_attention_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess) return noalloc_fail(err, err_len, FAK_NOALLOC_ECUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(e));
      g_noalloc_ptr[dev] = static_cast<float*>(p);
    }
    pw = g_noalloc_ptr[dev];
  }
  // partial outputs [slots, D] then (max, sum) pairs [slots] -- the layout the allocating path uses
  float2* pml = pw ? reinterpret_cast<float2*>(pw + slots * D) : nullptr;
  float2* dp = reinterpret_cast<float2*>(ds);
  const float scale_log2 = (1.0f / sqrtf((float)D)) * 1.4426950408889634f;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(Hkv, B, (unsigned)n_split);
  cfg.blockDim = dim3(128);
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  const __nv_bfloat16* kc = static_cast<const __nv_bfloat16*>(k_cache);
  const __nv_bfloat16* vc = static_cast<const __nv_bfloat16*>(v_cache);
  if (D == 128) {
    size_t smem = std::max(sizeof(DecodeSmem<128>), (size_t)(4 * 16 * 128 + 4 * 16 * 2) * 4);
    cfg.dynamicSmemBytes = smem;
    e = cudaFuncSetAttribute(k_decode_attn<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      e = cudaLaunchKernelEx(&cfg, k_decode_attn<128>, q, kc, vc, block_table, bt_stride, ctx_len, H, Hkv, n_split,
                             pages_per_split, scale_log2, pw, pml, out, qx, dp, ldo, nullptr, nullptr, 0, 0,
                             nullptr, 0, n_split, 0.f, 0.f, (const float*)nullptr);
  } else {
    size_t smem = std::max(sizeof(DecodeSmem<64>), (size_t)(4 * 16 * 64 + 4 * 16 * 2) * 4);
    cfg.dynamicSmemBytes = smem;
    e = cudaFuncSetAttribute(k_decode_attn<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e == cudaSuccess)
      e = cudaLaunchKernelEx(&cfg, k_decode_attn<64>, q, kc, vc, block_table, bt_stride, ctx_len, H, Hkv, n_split,
                             pages_per_split, scale_log2, pw, pml, out, qx, dp, ldo, nullptr, nullptr, 0, 0,
                             nullptr, 0, n_split, 0.f, 0.f, (const float*)nullptr);
  }
  if (e != cudaSuccess) return noalloc_fail(err, err_len, FAK_NOALLOC_ECUDA, "decode attention launch: %s", cudaGetErrorString(e));
  if (n_split > 1) {
    cudaLaunchConfig_t c2 = {};
    c2.gridDim = dim3(B, H);
    c2.blockDim = dim3(128);
    c2.stream = static_cast<cudaStream_t>(stream);
    if (D == 128)
      e = cudaLaunchKernelEx(&c2, k_decode_combine<128>, (const float*)pw, (const float2*)pml, H, n_split, out, qx,
                             dp, ldo, ctx_len, 0, (const int*)nullptr, 0, n_split, pages_per_split,
                             (const float*)nullptr);
    else
      e = cudaLaunchKernelEx(&c2, k_decode_combine<64>, (const float*)pw, (const float2*)pml, H, n_split, out, qx,
                             dp, ldo, ctx_len, 0, (const int*)nullptr, 0, n_split, pages_per_split,
                             (const float*)nullptr);
    if (e != cudaSuccess) return noalloc_fail(err, err_len, FAK_NOALLOC_ECUDA, "decode combine launch: %s", cudaGetErrorString(e));
  }
  return FAK_NOALLOC_OK;
}
