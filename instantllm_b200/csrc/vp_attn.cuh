// Embedding of the pass rows and tree-masked grouped-query attention (device functions of the
// persistent pass kernel, 512 threads per CTA).
//
// embed_row replaces k_embed_prompt (Sources/Engine/Shaders.swift:180-190) and the next-row embed
// of k_commit_spec (:413-417); it also validates the tree buffer and publishes the pass geometry
// (RowInfo) that every later stage reads.
//
// attn_unit replaces k_attention (Shaders.swift:876-958). Row t of a pass attends, in
// sequential-decode order, to its virtual sequence [cached slots 0..pos-1, then its ancestors in
// depth order, itself last]: exactly the keys the same token sees when the accepted path is decoded
// one token at a time. The sequence is cut into fixed 64-position chunks (flash-decoding partials:
// max, exp-sum, weighted V), combined in chunk order by the last chunk to finish. Chunk boundaries
// depend only on the virtual length, never on the pass shape, so a row's result is bit-identical in
// a 16-row tree pass and in a 1-row pass.
#pragma once
#include "vp_common.cuh"

namespace vp {

constexpr int PASS_THREADS = CONS_THREADS;

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

struct EmbedArgs {
  const uint8_t* E;
  const float* ln1;        // layer-0 input_layernorm weight
  const int32_t* prompt;   // prefill: token ids of this chunk (device); null for a verify pass
  int chunk_n;             // prefill: rows of this chunk
  int chunk_start;         // prefill: offset of the chunk in the prompt
  int total_n;             // prefill: prompt length
};

// Row t of the pass (t < 16; one CTA per row): validates the tree / prompt, embeds the row into x,
// writes its layer-0 QKV input (x * ln1 in act-block order) and its RMSNorm partials. The CTA of
// row 0 publishes RowInfo and the pass fields of the state. Zeros for padding rows.
template <int FMT>
__device__ void embed_row(const EmbedArgs& p, const Scratch& s, int t) {
  vp_state* st = s.st;
  const int tid = threadIdx.x;
  __shared__ int sTok, sN, sLive;
  __shared__ int sDepth[ROWS], sPar[ROWS];
  __shared__ float sPart[HRB];
  if (tid == 0) {
    int live = __ldcg(&st->done) == 0, err = 0, n, pos;
    if (p.prompt) {
      n = p.chunk_n;
      pos = __ldcg(&st->pos) + p.chunk_start;
      for (int i = 0; i < ROWS; ++i) { sDepth[i] = i; sPar[i] = i - 1; }
      if (n < 1 || n > ROWS) err |= VP_DEV_ERR_TREE;
      for (int i = 0; i < n && !err; ++i)
        if (p.prompt[i] < 0 || p.prompt[i] >= s.vocab) err |= VP_DEV_ERR_TREE;
      sTok = (!err && t < n) ? p.prompt[t] : 0;
    } else {
      n = s.tree[VP_TR_N];
      pos = __ldcg(&st->pos);
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
      sTok = t == 0 ? __ldcg(&st->last_token) : ((!err && t < n) ? s.tree[VP_TR_TOK + t] : 0);
      if (sTok < 0 || sTok >= s.vocab) err |= VP_DEV_ERR_TREE;
    }
    if (!err && (pos < 0 || pos + n > s.max_ctx)) err |= VP_DEV_ERR_CTX;
    if (err) live = 0;
    sN = n;
    sLive = live;
    if (t == 0) {
      if (err && __ldcg(&st->done) == 0) set_error(st, err);
      RowInfo* ri = s.ri;
      ri->n = n;
      ri->pos = pos;
      ri->mode = p.prompt ? 1 : 0;
      ri->live = live;
      for (int r = 0; r < ROWS; ++r) {
        const int dr = (r < n && !err) ? sDepth[r] : 0;
        ri->depth[r] = dr;
        int cur = r;
        for (int d = dr; d >= 0; --d) { ri->path[r][d] = cur; cur = cur > 0 ? sPar[cur] : 0; }
      }
      if (live) {
        st->n = n;
        st->mode = p.prompt ? 1 : 0;
        st->nver = p.prompt ? 1 : n;
        st->vrow0 = p.prompt ? n - 1 : 0;
        st->advance = p.prompt ? p.total_n : 0;
      }
    }
  }
  cons_sync();
  if (!sLive) return;
  const int n = sN, tok = sTok;
  // groups of 16 threads take row-blocks of 16 columns; both halves of a warp iterate equally often
  for (int rb = tid >> 4; rb < HRB; rb += PASS_THREADS / 16) {
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
  cons_sync();
  if (tid < HRB) s.ss[tid * 16 + t] = sPart[tid];
}

// ---------------------------------------------------------------------------------------------
// Attention

constexpr int GQ = NQ / NKV;            // 7 query heads per KV head
constexpr int ATT_TICKETS = 1024;       // offset of the attention arrival counters in tickets
constexpr int ATT_REC = GQ * (2 + HD);  // partial record of a chunk: per head m, l, o[64]
constexpr int ATT_SEG = 4;              // at most this many chunks per work unit (segment)
constexpr int ATT_PAD = 8;              // row padding (halves) against shared-memory bank conflicts

struct AttnSmem {
  float qs[GQ][HD];
  alignas(16) __half qh[2][8][HD + ATT_PAD];   // q * 0.125 as fp16 hi + lo parts, row 7 zero
  float sc[GQ][ATT_CHUNK + 4];
  alignas(16) __half kv[2][2][ATT_CHUNK][HD + ATT_PAD];  // [buffer][K, V][position][dim]
  int slots[ATT_SEG][ATT_CHUNK];
  float rec[ATT_SEG][ATT_REC];  // this segment's chunk partials
  int last;
};

// K/V double buffers double as the staging area of a row's chunk records in the combine.
constexpr int ATT_MAX_REC_STAGED = (int)(sizeof(__half) * 2 * 2 * ATT_CHUNK * (HD + ATT_PAD) / (ATT_REC * 4));

__device__ __forceinline__ int attn_chunks(const RowInfo* ri, int t, int pos) {
  return (pos + ri->depth[t] + 1 + ATT_CHUNK - 1) / ATT_CHUNK;
}
// Chunks per work unit: enough units to occupy `ctas` CTAs, at most ATT_SEG. The chunk records and
// their combine do not depend on how chunks are grouped into units, so this is free to follow the
// pass shape.
__device__ __forceinline__ int attn_segsize(const RowInfo* ri, int ctas) {
  int total = 0;
  for (int t = 0; t < ri->n; ++t) total += NKV * attn_chunks(ri, t, ri->pos);
  return min(ATT_SEG, max(1, (total + ctas - 1) / ctas));
}
__device__ __forceinline__ int attn_segs(int nch, int segsz) { return (nch + segsz - 1) / segsz; }

// Number of attention work units of a pass: (row, kv head, segment of <= segsz chunks).
__device__ int attn_units(const RowInfo* ri, int segsz) {
  const int n = ri->n, pos = ri->pos;
  int total = 0;
  for (int t = 0; t < n; ++t) total += NKV * attn_segs(attn_chunks(ri, t, pos), segsz);
  return total;
}

// Final output of (row t, kv head g) from the chunk partials in fixed chunk order:
// M = max m_c, O = sum o_c e^(m_c - M) / sum l_c e^(m_c - M).
template <bool GLOBAL>
__device__ __forceinline__ void attn_combine(const Scratch& s, const float* base, int nch, int t,
                                             int g) {
  for (int i = threadIdx.x; i < GQ * HD; i += PASS_THREADS) {
    const int h = i / HD, d = i % HD;
    auto ld = [&](const float* q) { return GLOBAL ? __ldcg(q) : *q; };
    float M = -INFINITY;
    for (int cc = 0; cc < nch; ++cc) M = fmaxf(M, ld(base + cc * ATT_REC + h * (2 + HD)));
    float O = 0.f, Ls = 0.f;
    for (int cc = 0; cc < nch; ++cc) {
      const float* r = base + cc * ATT_REC + h * (2 + HD);
      const float w = expf(ld(r) - M);
      Ls = fmaf(ld(r + 1), w, Ls);
      O = fmaf(ld(r + 2 + d), w, O);
    }
    s.act_a[act_index(t, (g * GQ + h) * HD + d)] = __float2half_rn(O / Ls);
  }
}

// One unit with PASS_THREADS threads: the chunks of one segment of (row t, kv head g), each a
// 64-position window of the row's virtual sequence. A row with one segment (virtual length <= 512)
// is combined right here; longer rows write chunk records and the segment that completes the row
// combines all of them (same formula, same chunk order).
__device__ void attn_unit(const Scratch& s, int layer, int max_chunks, int u, int segsz, AttnSmem& sm,
                          unsigned long long* trace = nullptr) {
  int ntr = 0;
  auto tstamp = [&]() {
    if (trace && threadIdx.x == 0 && ntr < 40) trace[ntr] = globaltimer();
    ++ntr;
  };
  tstamp();
  const RowInfo* ri = s.ri;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n = ri->n, pos = ri->pos;
  int t = 0, rem = u, nch = 1, nseg = 1;
  for (; t < n; ++t) {
    nch = attn_chunks(ri, t, pos);
    nseg = attn_segs(nch, segsz);
    if (rem < NKV * nseg) break;
    rem -= NKV * nseg;
  }
  const int g = rem / nseg, seg = rem % nseg;
  const int c0 = seg * segsz, c1 = min(nch, c0 + segsz);
  const int L = pos + ri->depth[t] + 1;
  const __half* kb = s.kc + (size_t)(layer * NKV + g) * s.max_ctx * HD;
  const __half* vb = s.vc + (size_t)(layer * NKV + g) * s.max_ctx * HD;
  // slots of every position of the segment (virtual position -> KV slot), no memory traffic
  for (int i = tid; i < (c1 - c0) * ATT_CHUNK; i += PASS_THREADS) {
    const int jv = c0 * ATT_CHUNK + i;
    sm.slots[i / ATT_CHUNK][i % ATT_CHUNK] =
        jv < pos ? jv : pos + ri->path[t][min(max(jv - pos, 0), ROWS - 1)];
  }
  cons_sync();
  // K and V rows of a chunk: 2 x 64 rows x 128 bytes = 1024 16-byte copies, two per thread, as
  // cp.async one chunk ahead (barriers do not wait for them); rows past the sequence are zeros.
  // evict-last keeps the KV cache resident in L2 against the streaming weights.
  const uint64_t kvpol = policy_evict_last();
  auto load_kv = [&](int ci, int buf) {
    const int cnt = min(L - (c0 + ci) * ATT_CHUNK, ATT_CHUNK);
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const int i = tid + k * PASS_THREADS;
      const int which = i / (ATT_CHUNK * 8), r = (i / 8) % ATT_CHUNK, part = i % 8;
      const int slot = r < cnt ? sm.slots[ci][r] : 0;
      cp_async16(&sm.kv[buf][which][r][part * 8], (which ? vb : kb) + (size_t)slot * HD + part * 8,
                 r < cnt ? 16u : 0u, kvpol);
    }
    cp_async_commit();
  };
  load_kv(0, 0);
  for (int i = tid; i < GQ * HD; i += PASS_THREADS)
    sm.qs[i / HD][i % HD] = __ldcg(s.q + t * H + (g * GQ + i / HD) * HD + i % HD);
  for (int c = c0; c < c1; ++c) {
    const int ci = c - c0, buf = ci & 1;
    const int j0 = c * ATT_CHUNK, cnt = min(L - j0, ATT_CHUNK);
    if (c + 1 < c1) {
      load_kv(ci + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    cons_sync();
    tstamp();
    // scores S = (q * 0.125) K^T on the tensor cores: warp w < 8 takes positions 8w..8w+7,
    // M = heads (7 of 16 rows used), K = 64 dims, q as fp16 hi + lo (near-fp32 product)
    if (c == c0) {
      for (int i = tid; i < 8 * HD; i += PASS_THREADS) {
        const int h = i / HD, d = i % HD;
        const float v = h < GQ ? sm.qs[h][d] * ATTN_SCALE : 0.f;
        const __half hi = __float2half_rn(v);
        sm.qh[0][h][d] = hi;
        sm.qh[1][h][d] = __float2half_rn(v - __half2float(hi));
      }
      cons_sync();
    }
    if (warp < 8) {
      const int gid = lane >> 2, t4 = lane & 3;
      float acc[2][4] = {};  // hi and lo parts of q: two independent chains, added at the end
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(&sm.kv[buf][0][warp * 8 + gid][ks * 16 + 2 * t4]);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(&sm.kv[buf][0][warp * 8 + gid][ks * 16 + 2 * t4 + 8]);
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          const uint32_t a0 = *reinterpret_cast<const uint32_t*>(&sm.qh[part][gid][ks * 16 + 2 * t4]);
          const uint32_t a2 = *reinterpret_cast<const uint32_t*>(&sm.qh[part][gid][ks * 16 + 2 * t4 + 8]);
          mma16816(acc[part], a0, 0u, a2, 0u, b0, b1);
        }
      }
      if (gid < GQ) {
        const int p0 = warp * 8 + 2 * t4;
        sm.sc[gid][p0] = p0 < cnt ? acc[0][0] + acc[1][0] : -INFINITY;
        sm.sc[gid][p0 + 1] = p0 + 1 < cnt ? acc[0][1] + acc[1][1] : -INFINITY;
      }
    }
    cons_sync();
    tstamp();
    // per-head max and exp-sum over the chunk (warp h, two positions per lane)
    if (warp < GQ) {
      const float v0 = sm.sc[warp][lane], v1 = sm.sc[warp][lane + 32];
      const float m = warp_max(fmaxf(v0, v1));
      const float e0 = lane < cnt ? expf(v0 - m) : 0.f;
      const float e1 = lane + 32 < cnt ? expf(v1 - m) : 0.f;
      sm.sc[warp][lane] = e0;
      sm.sc[warp][lane + 32] = e1;
      const float l = warp_sum(e0 + e1);
      if (lane == 0) { sm.rec[ci][warp * (2 + HD)] = m; sm.rec[ci][warp * (2 + HD) + 1] = l; }
    }
    cons_sync();
    tstamp();
    // weighted V: O = P V on the tensor cores: warp w < 8 takes dims 8w..8w+7, M = heads,
    // K = the chunk's 64 positions, P as fp16 hi + lo
    if (warp < 8) {
      const int gid = lane >> 2, t4 = lane & 3;
      float acc2[2][4] = {};  // hi and lo parts of P: two independent chains
      const int d = warp * 8 + gid;
#pragma unroll
      for (int ks = 0; ks < 4; ++ks)
#pragma unroll
        for (int part = 0; part < 2; ++part) {
          uint32_t a[2];
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int pp = ks * 16 + 2 * t4 + 8 * hh;
            float e0 = 0.f, e1 = 0.f;
            if (gid < GQ) { e0 = sm.sc[gid][pp]; e1 = sm.sc[gid][pp + 1]; }
            __half h0 = __float2half_rn(e0), h1 = __float2half_rn(e1);
            if (part) {
              h0 = __float2half_rn(e0 - __half2float(h0));
              h1 = __float2half_rn(e1 - __half2float(h1));
            }
            a[hh] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
          }
          const int pb = ks * 16 + 2 * t4;
          const uint32_t b0 = (uint32_t)__half_as_ushort(sm.kv[buf][1][pb][d]) |
                              ((uint32_t)__half_as_ushort(sm.kv[buf][1][pb + 1][d]) << 16);
          const uint32_t b1 = (uint32_t)__half_as_ushort(sm.kv[buf][1][pb + 8][d]) |
                              ((uint32_t)__half_as_ushort(sm.kv[buf][1][pb + 9][d]) << 16);
          mma16816(acc2[part], a[0], 0u, a[1], 0u, b0, b1);
        }
      if (gid < GQ) {
        sm.rec[ci][gid * (2 + HD) + 2 + warp * 8 + 2 * t4] = acc2[0][0] + acc2[1][0];
        sm.rec[ci][gid * (2 + HD) + 2 + warp * 8 + 2 * t4 + 1] = acc2[0][1] + acc2[1][1];
      }
    }
    cons_sync();
  }
  tstamp();
  if (nseg == 1) {
    attn_combine<false>(s, &sm.rec[0][0], nch, t, g);
    cons_sync();
    tstamp();
    return;
  }
  float* base = s.att_part + (size_t)(t * NKV + g) * max_chunks * ATT_REC;
  for (int i = tid; i < (c1 - c0) * ATT_REC; i += PASS_THREADS) base[c0 * ATT_REC + i] = (&sm.rec[0][0])[i];
  __threadfence();
  cons_sync();
  if (tid == 0) sm.last = atomicAdd(s.tickets + ATT_TICKETS + t * NKV + g, 1) == nseg - 1;
  cons_sync();
  if (sm.last) {
    __threadfence();
    // all chunk records of the row into shared memory in one coalesced round trip (they fit: the
    // K/V buffers are free now), then the combine reads shared memory only
    if (nch <= ATT_MAX_REC_STAGED) {
      float* recs = reinterpret_cast<float*>(&sm.kv[0][0][0][0]);
      for (int i = tid; i < nch * ATT_REC; i += PASS_THREADS) recs[i] = __ldcg(base + i);
      cons_sync();
      attn_combine<false>(s, recs, nch, t, g);
    } else {
      attn_combine<true>(s, base, nch, t, g);  // long rows: read the records in place
    }
    if (tid == 0) s.tickets[ATT_TICKETS + t * NKV + g] = 0;
  }
  cons_sync();
}

}  // namespace vp
