// Embedding of the pass rows and tree-masked grouped-query attention.
//
// k_embed replaces k_embed_prompt (Sources/Engine/Shaders.swift:180-190) and the next-row embed of
// k_commit_spec (:413-417): it also validates the tree buffer and publishes the pass geometry
// (RowInfo) that every later kernel reads.
//
// k_attention replaces k_attention (Shaders.swift:876-958). Row t of a pass attends, in
// sequential-decode order, to the virtual sequence [cached slots 0..pos-1, then its ancestors in
// depth order, itself last]: exactly the keys the same token would see if the accepted path had
// been decoded one token at a time. Work is split into fixed 64-position chunks of that virtual
// sequence (flash-decoding partials: max, sum, weighted V), combined in chunk order by the last
// chunk to finish. Chunk boundaries depend only on the virtual length, never on the pass shape,
// so a row's result is bit-identical in a 16-row tree pass and in a 1-row pass.
#pragma once
#include "vp_common.cuh"

namespace vp {

// Dequantised embedding value of (row tok, column k) read from the packed tile layout.
template <int FMT>
__device__ __forceinline__ float embed_value(const uint8_t* E, int tok, int k) {
  constexpr int TB = tile_bytes(FMT);
  const int rb = tok >> 4, r = tok & 15, g = r & 7, upper = r >> 3;
  const int G = k >> 6, kk = k & 63, j = kk >> 4, c = kk & 15;
  const int t4 = (c & 7) >> 1, reg = c >> 3, hi = c & 1;
  const int lane = g * 4 + t4, a = reg * 2 + upper;
  const uint8_t* tile = E + ((size_t)rb * (H / GS) + G) * TB;
  if constexpr (FMT == VP_FMT_Q4) {
    const uint32_t w = *reinterpret_cast<const uint32_t*>(tile + lane * 16 + j * 4);
    const float q = (float)((w >> ((hi ? 16 : 0) + 4 * a)) & 15u);
    const float2 sb = __half22float2(*reinterpret_cast<const __half2*>(tile + 512 + (g * 2 + upper) * 4));
    return __fadd_rn(__fmul_rn(sb.x, q), sb.y);
  } else if constexpr (FMT == VP_FMT_Q8) {
    const int8_t q = *reinterpret_cast<const int8_t*>(tile + lane * 32 + j * 8 + (a >> 1) * 4 +
                                                      (a & 1) * 2 + hi);
    const float s = __half2float(*reinterpret_cast<const __half*>(tile + 1024 + (g * 2 + upper) * 2));
    return __fmul_rn(s, (float)q);
  } else {
    return __half2float(
        *reinterpret_cast<const __half*>(tile + lane * 64 + j * 16 + a * 4 + hi * 2));
  }
}

struct EmbedParams {
  const uint8_t* E;
  const float* ln1;        // layer-0 input_layernorm weight
  const int32_t* prompt;   // prefill: token ids of this chunk (device); null for a verify pass
  int chunk_n;             // prefill: rows of this chunk
  int chunk_start;         // prefill: offset of the chunk in the prompt
  int total_n;             // prefill: prompt length
  int last_chunk;          // prefill: this chunk ends the prompt (its last row is committed)
  Scratch s;
};

// grid (16), 256 threads: CTA t embeds row t (zeros for padding rows); CTA 0 publishes RowInfo.
template <int FMT>
__global__ void __launch_bounds__(256) k_embed(EmbedParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const Scratch& s = p.s;
  vp_state* st = s.st;
  const int t = blockIdx.x, tid = threadIdx.x;
  __shared__ int sTok, sN, sLive, sPos;
  __shared__ int sDepth[ROWS], sPar[ROWS];
  if (tid == 0) {
    int live = st->done == 0, err = 0, n, pos;
    if (p.prompt) {
      n = p.chunk_n;
      pos = st->pos + p.chunk_start;
      for (int i = 0; i < ROWS; ++i) { sDepth[i] = i; sPar[i] = i - 1; }
      sTok = t < n ? p.prompt[t] : 0;
      if (n < 1 || n > ROWS) err |= VP_DEV_ERR_TREE;
      for (int i = 0; i < n && !err; ++i)
        if (p.prompt[i] < 0 || p.prompt[i] >= s.vocab) err |= VP_DEV_ERR_TREE;
    } else {
      n = s.tree[VP_TR_N];
      pos = st->pos;
      if (n < 1 || n > ROWS) err |= VP_DEV_ERR_TREE;
      for (int i = 0; i < ROWS && !err; ++i) {
        sDepth[i] = s.tree[VP_TR_DEPTH + i];
        sPar[i] = s.tree[VP_TR_PARENT + i];
      }
      if (!err) {
        if (sDepth[0] != 0) err |= VP_DEV_ERR_TREE;
        for (int i = 1; i < n; ++i) {
          const int pa = sPar[i];
          if (pa < 0 || pa >= i || sDepth[i] != sDepth[pa] + 1) err |= VP_DEV_ERR_TREE;
          const int tk = s.tree[VP_TR_TOK + i];
          if (tk < 0 || tk >= s.vocab) err |= VP_DEV_ERR_TREE;
        }
      }
      sTok = t == 0 ? st->last_token : (t < n ? s.tree[VP_TR_TOK + t] : 0);
      if (sTok < 0 || sTok >= s.vocab) err |= VP_DEV_ERR_TREE;
    }
    if (!err && (pos < 0 || pos + n > s.max_ctx)) err |= VP_DEV_ERR_CTX;
    if (err) live = 0;
    sN = n; sLive = live; sPos = pos;
    if (t == 0) {
      if (err && st->done == 0) set_error(st, err);
      RowInfo* ri = s.ri;
      ri->n = n; ri->pos = pos; ri->mode = p.prompt ? 1 : 0; ri->live = live;
      for (int r = 0; r < ROWS; ++r) {
        const int dr = (r < n && !err) ? sDepth[r] : 0;
        ri->depth[r] = dr;
        int cur = r;
        for (int d = dr; d >= 0; --d) { ri->path[r][d] = cur; cur = cur > 0 ? sPar[cur] : 0; }
      }
      if (live) {
        st->n = n;
        if (p.prompt) {
          st->mode = 1;
          st->nver = 1;
          st->vrow0 = n - 1;
          st->advance = p.total_n;
        } else {
          st->mode = 0;
          st->nver = n;
          st->vrow0 = 0;
          st->advance = 0;
        }
      }
    }
  }
  __syncthreads();
  if (!sLive) return;
  const int n = sN, tok = sTok;
  __shared__ float sPart[HRB];
  // Row t of x, of the layer-0 QKV input (x * ln1 in act-block order) and the RMSNorm partials.
  for (int rb = tid >> 4; rb < HRB; rb += 16) {
    const int k = rb * 16 + (tid & 15);
    float v = 0.f;
    if (t < n) v = embed_value<FMT>(p.E, tok, k);
    s.x[t * H + k] = v;
    s.act_h[act_index(t, k)] = __float2half_rn(v * p.ln1[k]);
    float sq = v * v;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o, 16);
    if ((tid & 15) == 0) sPart[rb] = sq;
  }
  __syncthreads();
  if (tid < HRB) s.ss[tid * 16 + t] = sPart[tid];
}

// ---------------------------------------------------------------------------------------------
// Attention

constexpr int ATT_THREADS = 256;
constexpr int GQ = NQ / NKV;  // 7 query heads per KV head
constexpr int ATT_TICKETS = 1024;  // offset of the attention arrival counters in Scratch::tickets

struct AttnParams {
  int layer;
  int max_chunks;   // chunks per (row, kv head) slot in att_part
  Scratch s;
};

// Partial record of one (row, kv head, chunk): per head m, l, o[64].
constexpr int ATT_REC = GQ * (2 + HD);

__global__ void __launch_bounds__(ATT_THREADS) k_attention(AttnParams p) {
  pdl_wait();
  pdl_launch_dependents();
  const Scratch& s = p.s;
  const RowInfo* ri = s.ri;
  if (!ri->live) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = ri->n, pos = ri->pos;
  __shared__ float qs[GQ][HD];
  __shared__ float sc[GQ][ATT_CHUNK];
  __shared__ int slots[ATT_CHUNK];
  __shared__ float sm[GQ], sl[GQ];
  __shared__ int sLast;

  // Units ordered by (row, kv head, chunk).
  int nch[ROWS];
  int total = 0;
  for (int t = 0; t < ROWS; ++t) {
    nch[t] = t < n ? (pos + ri->depth[t] + 1 + ATT_CHUNK - 1) / ATT_CHUNK : 0;
    total += 2 * nch[t];
  }
  for (int u = blockIdx.x; u < total; u += gridDim.x) {
    int t = 0, rem = u;
    while (rem >= 2 * nch[t]) { rem -= 2 * nch[t]; ++t; }
    const int g = rem / nch[t], c = rem % nch[t];
    const int L = pos + ri->depth[t] + 1;
    const int j0 = c * ATT_CHUNK, cnt = min(L - j0, ATT_CHUNK);
    const __half* kb = s.kc + (size_t)(p.layer * NKV + g) * s.max_ctx * HD;
    const __half* vb = s.vc + (size_t)(p.layer * NKV + g) * s.max_ctx * HD;
    for (int i = tid; i < GQ * HD; i += ATT_THREADS)
      qs[i / HD][i % HD] = s.q[t * H + (g * GQ + i / HD) * HD + i % HD];
    if (tid < ATT_CHUNK) {
      const int jv = j0 + tid;
      slots[tid] = jv < pos ? jv : pos + ri->path[t][min(jv - pos, ROWS - 1)];
    }
    __syncthreads();
    // Scores: 4 threads per position, 16 dims each, fixed-order combine.
    {
      const int pp = tid >> 2, part = tid & 3;
      float a[GQ];
#pragma unroll
      for (int h = 0; h < GQ; ++h) a[h] = 0.f;
      if (pp < cnt) {
        const __half2* kr = reinterpret_cast<const __half2*>(kb + (size_t)slots[pp] * HD + part * 16);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 kv = __half22float2(kr[i]);
#pragma unroll
          for (int h = 0; h < GQ; ++h)
            a[h] = fmaf(qs[h][part * 16 + 2 * i + 1], kv.y, fmaf(qs[h][part * 16 + 2 * i], kv.x, a[h]));
        }
      }
#pragma unroll
      for (int h = 0; h < GQ; ++h) {
        float v = a[h];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        if (part == 0) sc[h][pp] = pp < cnt ? v * ATTN_SCALE : -INFINITY;
      }
    }
    __syncthreads();
    // Per-head max and exp-sum over the chunk (warp h, two positions per lane).
    if (warp < GQ) {
      const float v0 = sc[warp][lane], v1 = sc[warp][lane + 32];
      const float m = warp_max(fmaxf(v0, v1));
      const float e0 = lane < cnt ? expf(v0 - m) : 0.f;
      const float e1 = lane + 32 < cnt ? expf(v1 - m) : 0.f;
      sc[warp][lane] = e0;
      sc[warp][lane + 32] = e1;
      const float l = warp_sum(e0 + e1);
      if (lane == 0) { sm[warp] = m; sl[warp] = l; }
    }
    __syncthreads();
    // Weighted V: thread (d, head set {hg, hg+4}), positions in order.
    {
      const int d = tid & 63, hg = tid >> 6;
      float o0 = 0.f, o1 = 0.f;
      for (int pp = 0; pp < cnt; ++pp) {
        const float v = __half2float(vb[(size_t)slots[pp] * HD + d]);
        o0 = fmaf(sc[hg][pp], v, o0);
        if (hg + 4 < GQ) o1 = fmaf(sc[hg + 4][pp], v, o1);
      }
      float* rec = s.att_part + ((size_t)(t * NKV + g) * p.max_chunks + c) * ATT_REC;
      rec[hg * (2 + HD) + 2 + d] = o0;
      if (hg + 4 < GQ) rec[(hg + 4) * (2 + HD) + 2 + d] = o1;
      if (tid < GQ) {
        rec[tid * (2 + HD)] = sm[tid];
        rec[tid * (2 + HD) + 1] = sl[tid];
      }
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) sLast = atomicAdd(s.tickets + ATT_TICKETS + t * NKV + g, 1) == nch[t] - 1;
    __syncthreads();
    if (sLast) {
      __threadfence();
      const float* base = s.att_part + (size_t)(t * NKV + g) * p.max_chunks * ATT_REC;
      for (int i = tid; i < GQ * HD; i += ATT_THREADS) {
        const int h = i / HD, d = i % HD;
        float M = -INFINITY;
        for (int cc = 0; cc < nch[t]; ++cc) M = fmaxf(M, __ldcg(base + cc * ATT_REC + h * (2 + HD)));
        float O = 0.f, Ls = 0.f;
        for (int cc = 0; cc < nch[t]; ++cc) {
          const float* r = base + cc * ATT_REC + h * (2 + HD);
          const float w = expf(__ldcg(r) - M);
          Ls = fmaf(__ldcg(r + 1), w, Ls);
          O = fmaf(__ldcg(r + 2 + d), w, O);
        }
        s.act_a[act_index(t, (g * GQ + h) * HD + d)] = __float2half_rn(O / Ls);
      }
      if (tid == 0) s.tickets[ATT_TICKETS + t * NKV + g] = 0;
    }
    __syncthreads();
  }
}

}  // namespace vp
