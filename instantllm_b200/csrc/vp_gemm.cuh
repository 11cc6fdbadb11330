// Skinny GEMM for the verification pass: Y[16 tokens][rows] = X[16][K] * W[rows][K]^T with the
// weight as the MMA's M side (swap-AB) and the padded 16 token rows as N.
//
// Replaces the reference's k_g3_* kernels (Sources/Engine/Shaders.swift:1911-2053, 2245-2257) and
// the T-templated decode kernels (:1201-1364) with one B200 design:
//  * Weights stream from HBM with cp.async.bulk into a per-warp ring of shared-memory slots
//    (mbarrier completion, evict-first L2 policy), three chunks in flight per warp.
//  * q4 / q8 codes are unpacked with one shift and four logic ops per 8 weights into fp16
//    *subnormals* (code * 2^-24, exact), so the tensor core multiplies exact integer codes; the
//    affine dequantisation w = s*q + b is applied per 64-column group on the fp32 accumulator:
//    y += s * 2^24 * sum(q x) + b * sum(x)  (same algebra as Shaders.swift:1182, done exactly).
//  * Each warp owns whole 16-row blocks; K may be split across CTAs, and split partials are summed
//    in a fixed order by whichever warp arrives last (ticket counter), so every output row is a
//    fixed function of its inputs: identical for 1-row and 16-row passes (tree == sequential).
//  * Epilogues: QKV (RMSNorm scale, bias, RoPE by tree depth, KV-cache write), residual add (+ the
//    next RMSNorm's weighted fp16 input and sum-of-squares partials), SiLU(gate)*up, and lm_head
//    max/argmax per 16 vocabulary rows.
#pragma once
#include "vp_common.cuh"

namespace vp {

enum GemmMode { MODE_QKV = 0, MODE_RESID = 1, MODE_SILU = 2, MODE_ARGMAX = 3 };

constexpr int GEMM_WARPS = 8;
constexpr int GEMM_NST = 2;  // ring slots per warp

// Greedy argmax through one atomic max per row: the key orders by logit (an order-preserving
// unsigned encoding of the float), then by the lower id. A zero key means nothing was inserted.
struct ArgmaxKeys {
  unsigned long long best[16];
  unsigned done;  // CTAs finished
};
// NaN gets 0, below every number (-inf included): like the commit kernel's `v > best`, which never
// selects a NaN logit while a number exists.
__device__ __forceinline__ unsigned ordered_bits(float f) {
  if (f != f) return 0u;
  const unsigned u = __float_as_uint(f + 0.f);  // -0 -> +0: equal floats get equal keys
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ unsigned long long argmax_key(float v, int id) {
  return ((unsigned long long)ordered_bits(v) << 32) | (unsigned)(0x7fffffff - id);
}
__device__ __forceinline__ int argmax_key_id(unsigned long long k) {
  return 0x7fffffff - (int)(unsigned)(k & 0xffffffffu);
}

// k_gemm<ARGMAX> with keys: the CTA's best key per row, merged into the global keys once per CTA
// (one copy per CTA; cleared before gemm_cta's first barrier).
__shared__ unsigned long long gemm_cta_keys[16];

struct GemmParams {
  const uint8_t* w;      // packed tiles [nrb][ng]
  const __half* act;     // act blocks [ng]
  int nrb, ng, nsplit;   // row-blocks, K groups, K splits (CTAs of a split share its act blocks)
  int cg;                // groups per ring chunk
  int cps;               // CTAs per split
  int layer;
  // inputs of the fused epilogues
  const float* bias;     // QKV: [1152]
  const float* ss_in;    // QKV / SILU / ARGMAX: RMSNorm partials [HRB][16] of the GEMM input
  const float* wnext;    // RESID: weight of the RMSNorm that consumes the updated x
  float* ss_out;         // RESID: partials of the updated x
  __half* act_out;       // RESID: normed input of the next GEMM; SILU: down-proj input
  float* pval;           // ARGMAX
  int* pidx;
  float* dbg;            // ARGMAX: optional full logits [16][nrb*16]
  ArgmaxKeys* keys;      // ARGMAX: optional; instead of pval / pidx, each row's (logit, id) goes into
                         // an atomic max and the last CTA writes tokens[0 .. out_rows)
  int32_t* tokens;
  int out_rows;
  float* xs;             // RESID: x[16 tokens][16 dims] of the row-block kept in shared memory by
                         // the CTA that owns it (persistent kernel), or null to use global x
  uint64_t* act_ll_out;  // RESID (persistent kernel, O): flagged act blocks / partials instead of
  uint64_t* ss_ll_out;   // act_out / ss_out
  const uint64_t* act_ll_in;  // SILU (persistent kernel): flagged inputs instead of act / ss_in
  const uint64_t* ss_ll_in;
  uint32_t flag;         // flag of this launch and layer
  const unsigned* gate;  // persistent kernel: flagged inputs are polled once this arrival counter
  unsigned gate_target;  // reaches gate_target (every producer CTA wrote its words), or null
  uint64_t* part_ll_out;       // RESID, split down projection: this CTA's partial tile goes out as
  const uint64_t* part_ll_in;  // flagged words (second CTA) / is added to the one polled here (first)
  Scratch s;
};

__host__ inline size_t gemm_smem_bytes(int fmt, int ng, int nsplit, int cg) {
  const int ngs = (ng + nsplit - 1) / nsplit;
  size_t b = (size_t)ngs * 2048 + (size_t)ngs * 16 * 4 * (fmt_halves(fmt) ? 2 : 1) + 16 * 4;
  // act blocks, group sums (per 32-column half for q8g32), rscale
  b = (b + 127) & ~size_t(127);
  b += (size_t)GEMM_WARPS * GEMM_NST * cg * tile_bytes(fmt);
  b += 8 * (1 + GEMM_WARPS * GEMM_NST) + 128;
  return b;
}

// A fragments of one 16-column k-step from a lane's 32-bit word of a q4 tile.
__device__ __forceinline__ void q4_frags(uint32_t v, uint32_t (&a)[4]) {
  const uint32_t v8 = v >> 8;
  a[0] = v & 0x000F000Fu;   // row gid,   codes * 2^-24
  a[1] = v & 0x00F000F0u;   // row gid+8, codes * 2^-20
  a[2] = v8 & 0x000F000Fu;
  a[3] = v8 & 0x00F000F0u;
}

// Per-row (gid, gid+8) affine constants of a q4 tile from the lane's 8 bytes of its scale block:
// y += sf * acc + sb * X.
__device__ __forceinline__ void q4_fold(uint2 v, float (&sf)[2], float (&sb)[2]) {
  const float2 p0 = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
  const float2 p1 = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
  sf[0] = p0.x * 16777216.f; sb[0] = p0.y;   // codes of row gid are code * 2^-24
  sf[1] = p1.x * 1048576.f;  sb[1] = p1.y;   // codes of row gid+8 are code * 2^-20
}

template <int FMT>
__device__ __forceinline__ void load_a_frags(const uint8_t* tile, int lane, int j, uint32_t (&a)[4]) {
  if constexpr (FMT == VP_FMT_Q4) {
    q4_frags(reinterpret_cast<const uint32_t*>(tile + lane * 16)[j], a);
  } else if constexpr (fmt_is_q8(FMT)) {
    const uint2 v = reinterpret_cast<const uint2*>(tile + lane * 32)[j];
    const uint32_t u0 = v.x ^ 0x80808080u, u1 = v.y ^ 0x80808080u;  // q + 128 in 1..255
    a[0] = __byte_perm(u0, 0u, 0x5150);   // bytes 0,1 -> low bytes of two halves
    a[1] = __byte_perm(u0, 0u, 0x5352);
    a[2] = __byte_perm(u1, 0u, 0x5150);
    a[3] = __byte_perm(u1, 0u, 0x5352);
  } else {
    const uint4 v = reinterpret_cast<const uint4*>(tile + lane * 64)[j];
    a[0] = v.x; a[1] = v.y; a[2] = v.z; a[3] = v.w;
  }
}

// A fragments of all four k-steps of a tile in one go: the lane's codes are loaded with 128-bit
// shared-memory reads (q4: one, q8: two, f16: four), conflict-free across the warp.
template <int FMT>
__device__ __forceinline__ void load_a_frags_all(const uint8_t* tile, int lane, uint32_t (&a)[4][4]) {
  if constexpr (FMT == VP_FMT_Q4) {
    const uint4 v = *reinterpret_cast<const uint4*>(tile + lane * 16);
    q4_frags(v.x, a[0]);
    q4_frags(v.y, a[1]);
    q4_frags(v.z, a[2]);
    q4_frags(v.w, a[3]);
  } else if constexpr (fmt_is_q8(FMT)) {
    const uint4 v0 = *reinterpret_cast<const uint4*>(tile + lane * 32);
    const uint4 v1 = *reinterpret_cast<const uint4*>(tile + lane * 32 + 16);
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t u0 = w[2 * j] ^ 0x80808080u, u1 = w[2 * j + 1] ^ 0x80808080u;  // q + 128 in 1..255
      a[j][0] = __byte_perm(u0, 0u, 0x5150);
      a[j][1] = __byte_perm(u0, 0u, 0x5352);
      a[j][2] = __byte_perm(u1, 0u, 0x5150);
      a[j][3] = __byte_perm(u1, 0u, 0x5352);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 v = reinterpret_cast<const uint4*>(tile + lane * 64)[j];
      a[j][0] = v.x; a[j][1] = v.y; a[j][2] = v.z; a[j][3] = v.w;
    }
  }
}

// Per-row (gid, gid+8) and per-half constants of a q8g32 tile (one scale per 32 columns):
// y += sf[h] * acc[h] + sb[h] * X[h] for the halves h = 0 (columns 0..31) and 1 (32..63).
__device__ __forceinline__ void load_fold_halves(const uint8_t* tile, int gid, float (&sf)[2][2], float (&sb)[2][2]) {
  const uint2 v = *reinterpret_cast<const uint2*>(tile + 1024 + gid * 8);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const float2 p = __half22float2(*reinterpret_cast<const __half2*>(h ? &v.y : &v.x));
    sf[h][0] = p.x * 16777216.f; sb[h][0] = -128.f * p.x;   // (q + 128) * 2^-24, rows gid
    sf[h][1] = p.y * 16777216.f; sb[h][1] = -128.f * p.y;   // and gid + 8
  }
}

// Per-row (gid, gid+8) affine constants of one tile: y += sf * acc + sb * X.
template <int FMT>
__device__ __forceinline__ void load_fold(const uint8_t* tile, int gid, float (&sf)[2], float (&sb)[2]) {
  static_assert(!fmt_halves(FMT), "q8g32 tiles fold per half (load_fold_halves)");
  if constexpr (FMT == VP_FMT_Q4) {
    q4_fold(*reinterpret_cast<const uint2*>(tile + 512 + gid * 8), sf, sb);
  } else if constexpr (FMT == VP_FMT_Q8) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(tile + 1024 + gid * 4);
    const float2 p = __half22float2(*reinterpret_cast<const __half2*>(&v));
    sf[0] = p.x * 16777216.f; sb[0] = -128.f * p.x;   // (q + 128) * 2^-24
    sf[1] = p.y * 16777216.f; sb[1] = -128.f * p.y;
  } else {
    sf[0] = sf[1] = 1.f; sb[0] = sb[1] = 0.f;
  }
}

template <int MODE>
__device__ void gemm_epilogue(const GemmParams& p, int rb, float (&acc)[2][4], const float* rs,
                              int lane) {
  const Scratch& s = p.s;
  const RowInfo* ri = s.ri;
  const int n = ri->n;
  const int gid = lane >> 2, tid4 = lane & 3;
  if constexpr (MODE == MODE_QKV) {
    const int head = rb >> 2, d = (rb & 3) * 8 + gid;
    const float ba = p.bias[head * HD + d], bb = p.bias[head * HD + d + 32];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = nt * 8 + 2 * tid4 + e;
        if (t >= n) continue;
        float a = acc[nt][e] * rs[t] + ba;
        float b = acc[nt][2 + e] * rs[t] + bb;
        if (head < NQ + NKV) {
          const float2 cs = s.rope[(ri->pos + ri->depth[t]) * 32 + d];
          const float a2 = a * cs.x - b * cs.y;
          const float b2 = b * cs.x + a * cs.y;
          a = a2; b = b2;
        }
        if (head < NQ) {
          s.q[t * H + head * HD + d] = a;
          s.q[t * H + head * HD + d + 32] = b;
        } else {
          const int kvh = head < NQ + NKV ? head - NQ : head - NQ - NKV;
          __half* c = head < NQ + NKV ? s.kc : s.vc;
          __half* row = c + ((size_t)(p.layer * NKV + kvh) * s.max_ctx + ri->pos + t) * HD;
          row[d] = __float2half_rn(a);
          row[d + 32] = __float2half_rn(b);
        }
      }
  } else if constexpr (MODE == MODE_RESID) {
    const int d0 = rb * 16 + gid, d1 = d0 + 8;
    const float w0 = p.wnext[d0], w1 = p.wnext[d1];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = nt * 8 + 2 * tid4 + e;
        float v0 = 0.f, v1 = 0.f;
        if (t < n) {
          const float x0 = p.xs ? p.xs[t * 16 + gid] : __ldcg(s.x + t * H + d0);
          const float x1 = p.xs ? p.xs[t * 16 + gid + 8] : __ldcg(s.x + t * H + d1);
          v0 = x0 + acc[nt][e];
          v1 = x1 + acc[nt][2 + e];
          if (p.xs) {
            p.xs[t * 16 + gid] = v0;
            p.xs[t * 16 + gid + 8] = v1;
          }
          s.x[t * H + d0] = v0;
          s.x[t * H + d1] = v1;
        }
        p.act_out[act_index(t, d0)] = __float2half_rn(v0 * w0);
        p.act_out[act_index(t, d1)] = __float2half_rn(v1 * w1);
        float sq = v0 * v0 + v1 * v1;
        sq += __shfl_xor_sync(0xffffffffu, sq, 4);
        sq += __shfl_xor_sync(0xffffffffu, sq, 8);
        sq += __shfl_xor_sync(0xffffffffu, sq, 16);
        if (gid == 0) p.ss_out[rb * 16 + t] = sq;
      }
  } else if constexpr (MODE == MODE_SILU) {
    const int f = rb * 8 + gid;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = nt * 8 + 2 * tid4 + e;
        float h = 0.f;
        if (t < n) {
          const float g = acc[nt][e] * rs[t];
          const float u = acc[nt][2 + e] * rs[t];
          h = g / (1.f + expf(-g)) * u;
        }
        p.act_out[act_index(t, f)] = __float2half_rn(h);
      }
  } else {  // MODE_ARGMAX
    const int v0 = rb * 16 + gid, v1 = v0 + 8;
    const int V = p.nrb * 16;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = nt * 8 + 2 * tid4 + e;
        const float l0 = acc[nt][e] * rs[t], l1 = acc[nt][2 + e] * rs[t];
        if (p.dbg) {
          p.dbg[(size_t)t * V + v0] = l0;
          p.dbg[(size_t)t * V + v1] = l1;
        }
        float bv = l0;
        int bi = v0;
        if (l1 > bv) { bv = l1; bi = v1; }
#pragma unroll
        for (int o = 4; o < 32; o <<= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
          if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
        }
        if (gid == 0) {
          if (p.keys) {
            if (t < p.out_rows) atomicMax(gemm_cta_keys + t, argmax_key(bv, bi));
          } else {
            p.pval[(size_t)t * p.nrb + rb] = bv;
            p.pidx[(size_t)t * p.nrb + rb] = bi;
          }
        }
      }
  }
}

// One CTA's share of a GEMM launch. smem layout: [act blocks][group sums][rscale][ring][barriers].
template <int FMT, int MODE>
__device__ void gemm_cta(const GemmParams& p, uint8_t* smem, int cta) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tid4 = lane & 3;
  const int split = cta % p.nsplit, cin = cta / p.nsplit;
  const int g0 = split * p.ng / p.nsplit, g1 = (split + 1) * p.ng / p.nsplit;
  const int ngs_max = (p.ng + p.nsplit - 1) / p.nsplit;
  constexpr int TB = tile_bytes(FMT);

  uint8_t* sAct = smem;
  float* sX = reinterpret_cast<float*>(smem + (size_t)ngs_max * 2048);
  float* sRs = sX + ngs_max * 16 * (fmt_halves(FMT) ? 2 : 1);
  // same layout as gemm_smem_bytes: act blocks, group sums (two per group for q8g32), rscale
  size_t off = (size_t)ngs_max * 2048 + (size_t)ngs_max * 16 * 4 * (fmt_halves(FMT) ? 2 : 1) + 16 * 4;
  off = (off + 127) & ~size_t(127);
  uint8_t* ring = smem + off + (size_t)warp * GEMM_NST * p.cg * TB;
  off += (size_t)GEMM_WARPS * GEMM_NST * p.cg * TB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + off);
  uint64_t* barAct = bars;
  uint64_t* myBars = bars + 1 + warp * GEMM_NST;
  __shared__ int sOk;

  if (threadIdx.x == 0) {
    mbar_init(barAct, 1);
    for (int i = 0; i < GEMM_WARPS * GEMM_NST; ++i) mbar_init(bars + 1 + i, 1);
    fence_barrier_init();
    sOk = 1;
  }
  cta_sync();

  // This warp's row-blocks: cin*4 + warp, then strided by all warps of the split.
  const int rb_first = cin * GEMM_WARPS + warp, rb_stride = p.cps * GEMM_WARPS;
  const int nchunk_rb = (g1 - g0 + p.cg - 1) / p.cg;
  int my_nrb = 0;
  if (rb_first < p.nrb) my_nrb = (p.nrb - 1 - rb_first) / rb_stride + 1;
  const int total_chunks = my_nrb * nchunk_rb;
  const uint64_t pol = policy_evict_first();

  auto issue = [&](int ci) {
    const int rbi = ci / nchunk_rb, c = ci % nchunk_rb;
    const int rb = rb_first + rbi * rb_stride;
    const int ga = g0 + c * p.cg, gb = min(g1, ga + p.cg);
    const uint32_t bytes = (uint32_t)(gb - ga) * TB;
    const int slot = ci % GEMM_NST;
    mbar_arrive_expect_tx(myBars + slot, bytes);
    bulk_g2s(ring + (size_t)slot * p.cg * TB, p.w + ((size_t)rb * p.ng + ga) * TB, bytes,
             myBars + slot, pol);
  };

  // Weights do not depend on earlier kernels: start streaming them before waiting on those.
  int n_issued = min(GEMM_NST, total_chunks);  // identical in every lane of the warp
  if (lane == 0)
    for (int ci = 0; ci < n_issued; ++ci) issue(ci);
  pdl_launch_dependents();
  pdl_wait();

  const bool live = p.s.ri->live != 0;
  if (live) {
    if (threadIdx.x == 0) {
      const uint32_t bytes = (uint32_t)(g1 - g0) * 2048;
      mbar_arrive_expect_tx(barAct, bytes);
      bulk_g2s(sAct, p.act + (size_t)g0 * 1024, bytes, barAct, policy_evict_last());
    }
    if (MODE != MODE_RESID && threadIdx.x < 16)
      sRs[threadIdx.x] = rms_inv([&](int r) { return __ldcg(p.ss_in + r * 16 + threadIdx.x); });
    // every warp waits (warp-uniform) for the act blocks; a timeout is recorded, not acted on per lane
    const bool act_ok = mbar_wait_warp(barAct, 0);
    if (!act_ok && lane == 0) sOk = 0;
    // Group sums X[g][t] = sum of the group's 64 fp16 inputs of token t (exact products, fp32
    // accumulation) via a ones-matrix MMA.
    if (FMT != VP_FMT_F16 && act_ok) {
      const uint32_t ONE2 = 0x3C003C00u;
      for (int g = warp; g < g1 - g0; g += GEMM_WARPS) {
        constexpr int NH = fmt_halves(FMT) ? 2 : 1;
        float xs[NH][2][4] = {};
        const uint8_t* ab = sAct + (size_t)g * 2048;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 b = *reinterpret_cast<const uint4*>(ab + j * 512 + lane * 16);
          const int h = NH == 2 ? (j >> 1) : 0;
          mma16816(xs[h][0], ONE2, ONE2, ONE2, ONE2, b.x, b.y);
          mma16816(xs[h][1], ONE2, ONE2, ONE2, ONE2, b.z, b.w);
        }
        if (gid == 0) {
#pragma unroll
          for (int h = 0; h < NH; ++h) {
            float* xo = sX + (g * NH + h) * 16;
            xo[2 * tid4] = xs[h][0][0];
            xo[2 * tid4 + 1] = xs[h][0][1];
            xo[8 + 2 * tid4] = xs[h][1][0];
            xo[8 + 2 * tid4 + 1] = xs[h][1][1];
          }
        }
      }
    }
  }
  cta_sync();
  bool ok = live && sOk != 0;
  if (live && !ok && threadIdx.x == 0) set_error(p.s.st, VP_DEV_ERR_TIMEOUT);

  float acc[2][4];
  int n_waited = 0;
  for (int ci = 0; ok && ci < total_chunks; ++ci) {
    const int slot = ci % GEMM_NST;
    if (!mbar_wait_warp(myBars + slot, (ci / GEMM_NST) & 1)) {
      if (lane == 0) set_error(p.s.st, VP_DEV_ERR_TIMEOUT);
      ok = false;
      break;
    }
    n_waited = ci + 1;
    const int rbi = ci / nchunk_rb, c = ci % nchunk_rb;
    const int rb = rb_first + rbi * rb_stride;
    const int ga = g0 + c * p.cg, gb = min(g1, ga + p.cg);
    if (c == 0) {
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[nt][i] = 0.f;
    }
    const uint8_t* slotp = ring + (size_t)slot * p.cg * TB;
    for (int g = ga; g < gb; ++g) {
      const uint8_t* tile = slotp + (size_t)(g - ga) * TB;
      const uint8_t* ab = sAct + (size_t)(g - g0) * 2048;
      if constexpr (FMT == VP_FMT_F16) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          load_a_frags<FMT>(tile, lane, j, a);
          const uint4 b = *reinterpret_cast<const uint4*>(ab + j * 512 + lane * 16);
          mma16816(acc[0], a[0], a[1], a[2], a[3], b.x, b.y);
          mma16816(acc[1], a[0], a[1], a[2], a[3], b.z, b.w);
        }
      } else if constexpr (fmt_halves(FMT)) {
        // q8g32: the two 32-column halves accumulate and fold separately
        float ag[2][2][4] = {};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          load_a_frags<FMT>(tile, lane, j, a);
          const uint4 b = *reinterpret_cast<const uint4*>(ab + j * 512 + lane * 16);
          mma16816(ag[j >> 1][0], a[0], a[1], a[2], a[3], b.x, b.y);
          mma16816(ag[j >> 1][1], a[0], a[1], a[2], a[3], b.z, b.w);
        }
        float sf[2][2], sb[2][2];
        load_fold_halves(tile, gid, sf, sb);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const float* xg = sX + ((g - g0) * 2 + h) * 16;
          const float2 x0 = *reinterpret_cast<const float2*>(xg + 2 * tid4);
          const float2 x1 = *reinterpret_cast<const float2*>(xg + 8 + 2 * tid4);
          const float tx[2][2] = {{x0.x, x0.y}, {x1.x, x1.y}};
#pragma unroll
          for (int nt = 0; nt < 2; ++nt)
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int r = i >> 1;
              acc[nt][i] = fmaf(sf[h][r], ag[h][nt][i], fmaf(sb[h][r], tx[nt][i & 1], acc[nt][i]));
            }
        }
      } else {
        float ag[2][4] = {};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint32_t a[4];
          load_a_frags<FMT>(tile, lane, j, a);
          const uint4 b = *reinterpret_cast<const uint4*>(ab + j * 512 + lane * 16);
          mma16816(ag[0], a[0], a[1], a[2], a[3], b.x, b.y);
          mma16816(ag[1], a[0], a[1], a[2], a[3], b.z, b.w);
        }
        float sf[2], sb[2];
        load_fold<FMT>(tile, gid, sf, sb);
        const float* xg = sX + (g - g0) * 16;
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
    }
    __syncwarp();
    if (ci + GEMM_NST < total_chunks) {
      if (lane == 0) issue(ci + GEMM_NST);
      n_issued = ci + GEMM_NST + 1;
    }

    if (c == nchunk_rb - 1) {
      // Row-block done for this split.
      if (p.nsplit == 1) {
        gemm_epilogue<MODE>(p, rb, acc, sRs, lane);
      } else {
        float* part = p.s.part + ((size_t)rb * p.nsplit + split) * 256;
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = gid + 8 * (i >> 1), t = nt * 8 + 2 * tid4 + (i & 1);
            part[r * 16 + t] = acc[nt][i];
          }
        __threadfence();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(p.s.tickets + rb, 1) == p.nsplit - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          float sum[2][4] = {};
          for (int sp = 0; sp < p.nsplit; ++sp) {
            const float* pp = p.s.part + ((size_t)rb * p.nsplit + sp) * 256;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const int r = gid + 8 * (i >> 1), t = nt * 8 + 2 * tid4 + (i & 1);
                sum[nt][i] += (sp == split) ? acc[nt][i] : __ldcg(pp + r * 16 + t);
              }
          }
          if (lane == 0) p.s.tickets[rb] = 0;
          gemm_epilogue<MODE>(p, rb, sum, sRs, lane);
        }
      }
    }
  }
  // Every copy this warp issued must land before the CTA's shared memory is released.
  for (int ci = n_waited; ci < n_issued; ++ci)
    mbar_wait_bounded(myBars + ci % GEMM_NST, (ci / GEMM_NST) & 1);
  if (threadIdx.x == 0 && live) mbar_wait_bounded(barAct, 0);
}

template <int FMT, int MODE>
__global__ void __launch_bounds__(GEMM_WARPS * 32) k_gemm(GemmParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  if constexpr (MODE == MODE_ARGMAX)
    if (p.keys && threadIdx.x < 16) gemm_cta_keys[threadIdx.x] = 0ull;
  gemm_cta<FMT, MODE>(p, smem, blockIdx.x);
  if constexpr (MODE == MODE_ARGMAX) {
    if (p.keys) {  // the last CTA to finish writes the tokens (-1 after a device-side timeout)
      __shared__ bool sLast;
      cta_sync();
      if (threadIdx.x < p.out_rows && gemm_cta_keys[threadIdx.x])
        atomicMax(p.keys->best + threadIdx.x, gemm_cta_keys[threadIdx.x]);
      cta_sync();
      if (threadIdx.x == 0) {
        __threadfence();
        sLast = atomicAdd(&p.keys->done, 1u) == gridDim.x - 1;
      }
      cta_sync();
      if (sLast) {
        __threadfence();
        if (threadIdx.x < p.out_rows) {
          const unsigned long long k = atomicOr(p.keys->best + threadIdx.x, 0ull);
          p.tokens[threadIdx.x] = (p.s.st->err || !k) ? -1 : argmax_key_id(k);
        }
      }
    }
  }
}

}  // namespace vp
