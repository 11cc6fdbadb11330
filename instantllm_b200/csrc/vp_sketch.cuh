// Two-stage lm_head over a 2-bit sketch of the q4 embedding: the reference's k_lmh_sketch_T,
// k_lmh_tau and k_lmh_exact_T (Shaders.swift:1377-1523, Engine.swift:436-454), off by default
// there (useSketchHead, Engine.swift:34-39) because its argmax equals the full lm_head's only with
// overwhelming probability.
//
// Stage 1 scores every vocabulary row from the high two bits of its q4 codes:
//   w ~ s (4 hi + 1.5) + b        (the dropped low bits are ~uniform in 0..3: mean 1.5, var 1.25)
//   A = sum_g s_g (4 <hi_g, a_g> + 1.5 X_g) + b_g X_g,  sigma^2 = 1.25 sum_g s_g^2 |a_g|^2
// (a = the RMS-normed input, X_g / |a_g|^2 its sum / squared norm over the 64 columns of group g),
// and records, per 32-row vocabulary group, the max of A - K sigma and of A + K sigma. tau = the
// max over groups of the lower bound. Stage 2 recomputes exact q4 logits only in groups whose upper
// bound reaches tau; other groups report -inf, so the argmax equals the full lm_head's unless a
// residual exceeds K sigma.
//
// B200 layout: the sketch plane is packed, like the q4 weights, into 16 x 64 mma.sync A-fragment
// tiles of 256 bytes (lane L's 8 bytes at L*8), so stage 1 streams 256 + 64 bytes (sketch + the q4
// tile's scale block) per tile instead of 576, and feeds the codes to the tensor cores as fp16
// subnormals. Word w (0, 1) of a lane covers the k-steps j = 2w and 2w + 1; byte b of the word
// holds j = 2w + (b & 1), column parity hi = b >> 1, and in its bit pairs 0-1, 2-3, 4-5, 6-7 the
// codes of A registers a0 (row gid, column 16 j + 2 tid4 + hi), a1 (row gid + 8, same column),
// a2 (row gid, column + 8) and a3 (row gid + 8, column + 8). Masking a word with 0x00030003
// therefore yields a0 as two fp16 subnormals code * 2^-24, and 0x000C000C yields a1 as code * 2^-22:
// each row keeps one power-of-two scale across its four A registers.
//
// Stage 2 reproduces the arithmetic of the full lm_head (k_gemm<Q4, MODE_ARGMAX>: group sums by
// a ones-matrix MMA, per-group fold with fmaf in group order, the same rsqrt scale) row for row,
// so a recomputed logit is bit-identical to the full head's and the sketch head returns the same
// token whenever the bound holds.
#pragma once
#include <math.h>

#include "vp_gemm.cuh"

namespace vp {

constexpr int SK_TILE = 256;       // bytes of one packed 16 x 64 sketch tile
constexpr int SK_GROUP = 32;       // vocabulary rows per bound group (the reference's threadgroup)
constexpr int SK_WARPS = 8;
constexpr int SK_THREADS = SK_WARPS * 32;
constexpr int SK_NG = H / GS;      // 14 column groups of the hidden size

__host__ __device__ constexpr int sk_groups(int vocab) { return (vocab + SK_GROUP - 1) / SK_GROUP; }

// The per-call block both stages share, zeroed by k_sk_prep.
struct SketchSmall {
  unsigned tau[16];                // encoded max over groups of the lower bound (sk_enc)
  unsigned long long best[16];     // encoded (logit, id) argmax of the candidates (argmax_key)
  int cand0, cand_any;             // candidate groups of row 0, of any row
  unsigned done;                   // stage-2 CTAs finished
};

// Float max through unsigned atomics: the order-preserving encoding of vp_gemm.cuh (0 is below
// every float); (logit, id) keys are vp_gemm.cuh's argmax_key.
__device__ __forceinline__ unsigned sk_enc(float f) { return ordered_bits(f); }
__device__ __forceinline__ float sk_dec(unsigned u) {
  return __uint_as_float((u & 0x80000000u) ? (u & 0x7fffffffu) : ~u);
}

// Standard sketch plane hi [vocab][H/4] (byte c of a row: codes 4c .. 4c+3 >> 2, code 4c in bits
// 0-1; Convert.swift:150-158) -> packed tiles [vocab/16][14][256]. One thread per (tile, lane).
__global__ void k_pack_sketch(int vocab, const uint8_t* hi, uint8_t* out) {
  const long long ntiles = (long long)(vocab / 16) * SK_NG;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= ntiles * 32) return;
  const long long tileI = idx >> 5;
  const int lane = (int)(idx & 31), g = lane >> 2, t4 = lane & 3;
  const int rb = (int)(tileI / SK_NG), G = (int)(tileI % SK_NG);
  uint32_t words[2] = {0u, 0u};
  for (int w = 0; w < 2; ++w)
    for (int b = 0; b < 4; ++b) {
      const int j = 2 * w + (b & 1), par = b >> 1;
      uint32_t byte = 0;
      for (int i = 0; i < 4; ++i) {
        const int row = rb * 16 + g + 8 * (i & 1);
        const int col = G * GS + 16 * j + 8 * (i >> 1) + 2 * t4 + par;
        const uint32_t c = (hi[(size_t)row * (H / 4) + (col >> 2)] >> (2 * (col & 3))) & 3u;
        byte |= c << (2 * i);
      }
      words[w] |= byte << (8 * b);
    }
  reinterpret_cast<uint2*>(out + tileI * SK_TILE)[lane] = make_uint2(words[0], words[1]);
}

struct SketchParams {
  const uint8_t* sk;    // packed sketch tiles [nrb][14]
  const uint8_t* emb;   // packed q4 embedding tiles [nrb][14] (scale block at +512)
  const __half* act;    // act blocks [14] of half(x * final_norm), B-fragment order
  const float* ss;      // RMSNorm partials [HRB][16]
  float* bounds;        // [2][16][ngrp]: per-group max of A - K sigma, then of A + K sigma
  SketchSmall* small;   // tau, the running argmax keys, counters (zeroed by k_sk_prep)
  int32_t* tokens;      // [rows] result
  int32_t* ncand;       // optional [2] result: candidate groups of row 0, of any row
  int nrb, ngrp, rows;
  float k;
};

// Per CTA: act blocks into shared memory and the RMSNorm scale rs[t] (the full head's expression).
__device__ void sk_load_act(const SketchParams& p, uint8_t* sAct, float* sRs) {
  const uint4* src = reinterpret_cast<const uint4*>(p.act);
  uint4* dst = reinterpret_cast<uint4*>(sAct);
  for (int i = threadIdx.x; i < SK_NG * 2048 / 16; i += blockDim.x) dst[i] = __ldcg(src + i);
  if (threadIdx.x < 16) sRs[threadIdx.x] = rms_inv([&](int r) { return __ldcg(p.ss + r * 16 + threadIdx.x); });
}

// Stage 1. NT = 1 when rows <= 8 (one n8 half of the MMA), else 2. Each warp takes whole 32-row
// groups; the next row-block's 14 sketch words and scale blocks are in flight while the current one
// is computed.
template <int NT>
__global__ void __launch_bounds__(SK_THREADS, 2) k_sketch(SketchParams p) {
  __shared__ __align__(16) uint8_t sAct[SK_NG * 2048];
  __shared__ float sRs[16], sX[SK_NG][16], sXX[SK_NG][16];
  __shared__ unsigned sTau[16];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tid4 = lane & 3;

  // This warp's row-blocks, group by group. The 14 sketch words and scale blocks of the next
  // row-block are loaded into the registers of the current one as each is consumed, so a
  // row-block's loads stay in flight while the previous one is computed; the first row-block's
  // loads are issued before the act blocks are staged.
  const int wg = blockIdx.x * SK_WARPS + warp, wstride = gridDim.x * SK_WARPS;
  int n_my = 0;
  for (int grp = wg; grp < p.ngrp; grp += wstride) n_my += min(2, p.nrb - 2 * grp);
  auto rb_of = [&](int i) { return 2 * (wg + (i >> 1) * wstride) + (i & 1); };
  auto sk_ptr = [&](int i) { return p.sk + (size_t)rb_of(i) * SK_NG * SK_TILE + lane * 8; };
  auto sb_ptr = [&](int i) { return p.emb + (size_t)rb_of(i) * SK_NG * 576 + 512 + gid * 8; };

  uint2 skw[SK_NG], fold[SK_NG];
  if (n_my > 0) {
    const uint8_t* st = sk_ptr(0);
    const uint8_t* et = sb_ptr(0);
#pragma unroll
    for (int G = 0; G < SK_NG; ++G) {
      skw[G] = __ldcs(reinterpret_cast<const uint2*>(st + G * SK_TILE));
      fold[G] = __ldcs(reinterpret_cast<const uint2*>(et + G * 576));
    }
  }

  if (threadIdx.x < 16) sTau[threadIdx.x] = 0u;
  sk_load_act(p, sAct, sRs);
  cta_sync();
  // X[g][t], XX[g][t]: sum and squared norm of the 64 normed inputs of group g, token t, from the
  // lanes' B fragments (lane: columns 2 tid4, +1, +8, +9 of each k-step for tokens gid, gid + 8).
  for (int G = warp; G < SK_NG; G += SK_WARPS) {
    float s0 = 0.f, q0 = 0.f, s1 = 0.f, q1 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 b = *reinterpret_cast<const uint4*>(sAct + G * 2048 + j * 512 + lane * 16);
      const uint32_t w4[4] = {b.x, b.y, b.z, b.w};
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w4[r]));
        if (r < 2) { s0 += f.x + f.y; q0 = fmaf(f.x, f.x, fmaf(f.y, f.y, q0)); }
        else { s1 += f.x + f.y; q1 = fmaf(f.x, f.x, fmaf(f.y, f.y, q1)); }
      }
    }
#pragma unroll
    for (int o = 1; o < 4; o <<= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      q0 += __shfl_xor_sync(0xffffffffu, q0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
      q1 += __shfl_xor_sync(0xffffffffu, q1, o);
    }
    if (tid4 == 0) {
      sX[G][gid] = s0;
      sXX[G][gid] = q0;
      sX[G][gid + 8] = s1;
      sXX[G][gid + 8] = q1;
    }
  }
  cta_sync();

  float tmax[NT][2];  // this lane's tokens: running max of the lower bound over the warp's groups
  float glb[NT][2], gub[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) tmax[nt][0] = tmax[nt][1] = glb[nt][0] = glb[nt][1] = gub[nt][0] = gub[nt][1] = -INFINITY;
  for (int i = 0; i < n_my; ++i) {
    const bool more = i + 1 < n_my;
    const uint8_t* nst = sk_ptr(more ? i + 1 : i);
    const uint8_t* net = sb_ptr(more ? i + 1 : i);
    float A[NT][4], V[NT][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) A[nt][e] = V[nt][e] = 0.f;
#pragma unroll
    for (int G = 0; G < SK_NG; ++G) {
      const uint2 w = skw[G];
      const uint2 f = fold[G];
      if (more) {
        skw[G] = __ldcs(reinterpret_cast<const uint2*>(nst + G * SK_TILE));
        fold[G] = __ldcs(reinterpret_cast<const uint2*>(net + G * 576));
      }
      float ag[NT][4] = {};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t v = ((j >> 1) ? w.y : w.x) >> (8 * (j & 1));
        const uint32_t a0 = v & 0x00030003u, a1 = v & 0x000C000Cu;
        const uint32_t a2 = (v >> 4) & 0x00030003u, a3 = (v >> 4) & 0x000C000Cu;
        const uint8_t* ab = sAct + G * 2048 + j * 512 + lane * 16;
        if constexpr (NT == 1) {
          const uint2 b = *reinterpret_cast<const uint2*>(ab);
          mma16816(ag[0], a0, a1, a2, a3, b.x, b.y);
        } else {
          const uint4 b = *reinterpret_cast<const uint4*>(ab);
          mma16816(ag[0], a0, a1, a2, a3, b.x, b.y);
          mma16816(ag[1], a0, a1, a2, a3, b.z, b.w);
        }
      }
      const float2 sb0 = __half22float2(*reinterpret_cast<const __half2*>(&f.x));  // row gid
      const float2 sb1 = __half22float2(*reinterpret_cast<const __half2*>(&f.y));  // row gid + 8
      const float m[2] = {sb0.x * 67108864.f, sb1.x * 16777216.f};  // 4 s / 2^-24, 4 s / 2^-22
      const float c[2] = {fmaf(1.5f, sb0.x, sb0.y), fmaf(1.5f, sb1.x, sb1.y)};
      const float q[2] = {sb0.x * sb0.x, sb1.x * sb1.x};
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = e >> 1, t = nt * 8 + 2 * tid4 + (e & 1);
          A[nt][e] = fmaf(m[r], ag[nt][e], fmaf(c[r], sX[G][t], A[nt][e]));
          V[nt][e] = fmaf(q[r], sXX[G][t], V[nt][e]);
        }
    }
    // bounds of this row-block's 16 rows, max over rows (gid, gid + 8 in the lane; gid by shuffle)
    const bool first = (i & 1) == 0;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = nt * 8 + 2 * tid4 + e;
        const float rs = sRs[t];
        float lo = -INFINITY, up = -INFINITY;
#pragma unroll
        for (int r = 0; r < 2; ++r) {
          const float a = A[nt][2 * r + e] * rs, sg = rs * sqrtf(1.25f * V[nt][2 * r + e]);
          lo = fmaxf(lo, fmaf(-p.k, sg, a));
          up = fmaxf(up, fmaf(p.k, sg, a));
        }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          lo = fmaxf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
          up = fmaxf(up, __shfl_xor_sync(0xffffffffu, up, o));
        }
        glb[nt][e] = first ? lo : fmaxf(glb[nt][e], lo);
        gub[nt][e] = first ? up : fmaxf(gub[nt][e], up);
      }
    const int rb = rb_of(i);
    if (((i & 1) || rb + 1 >= p.nrb) && gid == 0) {  // group complete
      const int grp = rb >> 1;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = nt * 8 + 2 * tid4 + e;
          if (t < p.rows) {
            p.bounds[(size_t)t * p.ngrp + grp] = glb[nt][e];
            p.bounds[(size_t)(16 + t) * p.ngrp + grp] = gub[nt][e];
            tmax[nt][e] = fmaxf(tmax[nt][e], glb[nt][e]);
          }
        }
    }
  }
  if (gid == 0 && n_my > 0) {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = nt * 8 + 2 * tid4 + e;
        if (t < p.rows) atomicMax(&sTau[t], sk_enc(tmax[nt][e]));
      }
  }
  cta_sync();
  if (threadIdx.x < p.rows && sTau[threadIdx.x]) atomicMax(p.small->tau + threadIdx.x, sTau[threadIdx.x]);
}

// Stage 2. CTA c owns the groups [c * gpc, (c + 1) * gpc). Its warps sort them: a group whose upper
// bound reaches some row's tau goes into a shared list with its mask of candidate rows. If the list
// is not empty the CTA loads the act blocks, the RMSNorm scale and the group sums exactly as
// gemm_cta does for the full head, and its warps recompute the listed row-blocks with gemm_cta's
// q4 tile arithmetic (all 14 tiles of a row-block loaded before the first MMA). Each candidate row's
// best (logit, id) goes into an atomic max; a row for which the group is not a candidate takes no
// part (Shaders.swift:1475-1513 reports -inf there). The last CTA to finish writes the tokens.
constexpr int SK_MAX_GPC = 64;

__global__ void __launch_bounds__(SK_THREADS, 1) k_sk_exact(SketchParams p) {
  __shared__ __align__(16) uint8_t sAct[SK_NG * 2048];
  __shared__ __align__(16) float sX[SK_NG * 16];  // read as float2
  __shared__ float sRs[16], sTau[16];
  __shared__ int sList[SK_MAX_GPC];
  __shared__ unsigned sMask[SK_MAX_GPC];
  __shared__ int sN, sC0, sCA;
  __shared__ bool sLast;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, gid = lane >> 2, tid4 = lane & 3;
  SketchSmall* sm = p.small;
  const int gpc = (p.ngrp + gridDim.x - 1) / gridDim.x;
  const int g0 = blockIdx.x * gpc, g1 = min(p.ngrp, g0 + gpc);
  if (threadIdx.x < 16)
    sTau[threadIdx.x] = threadIdx.x < p.rows ? sk_dec(__ldcg(sm->tau + threadIdx.x)) : INFINITY;
  if (threadIdx.x == 0) sN = sC0 = sCA = 0;
  cta_sync();
  for (int grp = g0 + warp; grp < g1; grp += SK_WARPS) {
    const bool c = lane < p.rows && __ldcg(p.bounds + (size_t)(16 + lane) * p.ngrp + grp) >= sTau[lane & 15];
    const unsigned mask = __ballot_sync(0xffffffffu, c);
    if (mask != 0u && lane == 0) {
      const int k = atomicAdd(&sN, 1);
      sList[k] = grp;
      sMask[k] = mask;
      if (mask & 1u) atomicAdd(&sC0, 1);
      atomicAdd(&sCA, 1);
    }
  }
  cta_sync();
  const int n = sN;
  if (n > 0) {
    if (threadIdx.x == 0) {
      atomicAdd(&sm->cand0, sC0);
      atomicAdd(&sm->cand_any, sCA);
    }
    sk_load_act(p, sAct, sRs);
    cta_sync();
    {  // group sums X[g][t] by a ones-matrix MMA (gemm_cta's expression for q4)
      const uint32_t ONE2 = 0x3C003C00u;
      for (int g = warp; g < SK_NG; g += SK_WARPS) {
        float xs[2][4] = {};
        const uint8_t* ab = sAct + (size_t)g * 2048;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 b = *reinterpret_cast<const uint4*>(ab + j * 512 + lane * 16);
          mma16816(xs[0], ONE2, ONE2, ONE2, ONE2, b.x, b.y);
          mma16816(xs[1], ONE2, ONE2, ONE2, ONE2, b.z, b.w);
        }
        if (gid == 0) {
          float* xo = sX + g * 16;
          xo[2 * tid4] = xs[0][0];
          xo[2 * tid4 + 1] = xs[0][1];
          xo[8 + 2 * tid4] = xs[1][0];
          xo[8 + 2 * tid4 + 1] = xs[1][1];
        }
      }
    }
    cta_sync();
    for (int it = warp; it < 2 * n; it += SK_WARPS) {
      const int rb = 2 * sList[it >> 1] + (it & 1);
      if (rb >= p.nrb) continue;
      const unsigned mask = sMask[it >> 1];
      const uint8_t* row = p.emb + (size_t)rb * SK_NG * 576;
      uint4 cw[SK_NG];
      uint2 fw[SK_NG];
#pragma unroll
      for (int G = 0; G < SK_NG; ++G) {
        cw[G] = __ldcs(reinterpret_cast<const uint4*>(row + G * 576 + lane * 16));
        fw[G] = __ldcs(reinterpret_cast<const uint2*>(row + G * 576 + 512 + gid * 8));
      }
      float acc[2][4] = {};
#pragma unroll
      for (int G = 0; G < SK_NG; ++G) {
        const uint8_t* ab = sAct + (size_t)G * 2048;
        const uint32_t words[4] = {cw[G].x, cw[G].y, cw[G].z, cw[G].w};
        float ag[2][4] = {};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          q4_frags(words[j], a);
          const uint4 b = *reinterpret_cast<const uint4*>(ab + j * 512 + lane * 16);
          mma16816(ag[0], a[0], a[1], a[2], a[3], b.x, b.y);
          mma16816(ag[1], a[0], a[1], a[2], a[3], b.z, b.w);
        }
        float sf[2], sb[2];
        q4_fold(fw[G], sf, sb);
        const float* xg = sX + G * 16;
        const float2 x0 = *reinterpret_cast<const float2*>(xg + 2 * tid4);
        const float2 x1 = *reinterpret_cast<const float2*>(xg + 8 + 2 * tid4);
        const float tx[2][2] = {{x0.x, x0.y}, {x1.x, x1.y}};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = i >> 1;
            acc[nt][i] = fmaf(sf[r], ag[nt][i], fmaf(sb[r], tx[nt][i & 1], acc[nt][i]));
          }
      }
      const int v0 = rb * 16 + gid, v1 = v0 + 8;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = nt * 8 + 2 * tid4 + e;
          const float l0 = acc[nt][e] * sRs[t], l1 = acc[nt][2 + e] * sRs[t];
          float bv = l0;
          int bi = v0;
          if (l1 > bv) { bv = l1; bi = v1; }
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
          }
          if (gid == 0 && ((mask >> t) & 1u)) atomicMax(sm->best + t, argmax_key(bv, bi));
        }
    }
  }
  // the last CTA writes the tokens and the candidate counts (the barrier orders the CTA's atomics
  // before thread 0's fence and ticket)
  cta_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    sLast = atomicAdd(&sm->done, 1u) == gridDim.x - 1;
  }
  cta_sync();
  if (sLast) {
    __threadfence();
    if (threadIdx.x < p.rows) {
      const unsigned long long k = atomicOr(sm->best + threadIdx.x, 0ull);
      p.tokens[threadIdx.x] = k ? argmax_key_id(k) : -1;
    }
    if (threadIdx.x == 0 && p.ncand) {
      p.ncand[0] = atomicOr(&sm->cand0, 0);
      p.ncand[1] = atomicOr(&sm->cand_any, 0);
    }
  }
}

}  // namespace vp

