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
  } else if constexpr (FMT == VP_FMT_Q8G32) {
    const int8_t q = *reinterpret_cast<const int8_t*>(tile + lane * 32 + j * 8 + (a >> 1) * 4 +
                                                      (a & 1) * 2 + hi);
    const int half = kk >> 5;  // scale of the 32-column half
    const float s = __half2float(*reinterpret_cast<const __half*>(tile + 1024 + (g * 4 + half * 2 + upper) * 2));
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
  __shared__ int sIn[VP_TREE_INTS + 3];  // the tree buffer (or the prompt chunk), done, pos, last token
  // every input in one parallel round trip; the validation below then reads shared memory only
  if (p.prompt) {
    if (tid < p.chunk_n && tid < ROWS) sIn[tid] = p.prompt[tid];
  } else if (tid < VP_TREE_INTS) {
    sIn[tid] = s.tree[tid];
  }
  if (tid == VP_TREE_INTS) sIn[tid] = __ldcg(&st->done);
  if (tid == VP_TREE_INTS + 1) sIn[tid] = __ldcg(&st->pos);
  if (tid == VP_TREE_INTS + 2) sIn[tid] = __ldcg(&st->last_token);
  cons_sync();
  if (tid == 0) {
    int live = sIn[VP_TREE_INTS] == 0, err = 0, n, pos;
    if (p.prompt) {
      n = p.chunk_n;
      pos = sIn[VP_TREE_INTS + 1] + p.chunk_start;
      for (int i = 0; i < ROWS; ++i) { sDepth[i] = i; sPar[i] = i - 1; }
      if (n < 1 || n > ROWS) err |= VP_DEV_ERR_TREE;
      for (int i = 0; i < n && !err; ++i)
        if (sIn[i] < 0 || sIn[i] >= s.vocab) err |= VP_DEV_ERR_TREE;
      sTok = (!err && t < n) ? sIn[t] : 0;
    } else {
      n = sIn[VP_TR_N];
      pos = sIn[VP_TREE_INTS + 1];
      if (n < 1 || n > ROWS) err |= VP_DEV_ERR_TREE;
      for (int i = 0; i < ROWS && !err; ++i) {
        sDepth[i] = sIn[VP_TR_DEPTH + i];
        sPar[i] = sIn[VP_TR_PARENT + i];
      }
      if (!err) {
        if (sDepth[0] != 0) err |= VP_DEV_ERR_TREE;
        for (int i = 1; i < n; ++i) {
          const int pa = sPar[i];
          if (pa < 0 || pa >= i || sDepth[i] != sDepth[pa] + 1) err |= VP_DEV_ERR_TREE;
          const int tk = sIn[VP_TR_TOK + i];
          if (tk < 0 || tk >= s.vocab) err |= VP_DEV_ERR_TREE;
        }
      }
      sTok = t == 0 ? sIn[VP_TREE_INTS + 2] : ((!err && t < n) ? sIn[VP_TR_TOK + t] : 0);
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

// Attention
//
// Records: the virtual sequence of row t is cut into fixed 32-position sub-chunks; each
// (row, query head, sub-chunk) gets a record (max, exp-sum, unnormalised o[64]) and the output is
// the combine of the row's records in sub-chunk order. Sub-chunk boundaries depend only on virtual
// positions, so a row's output is bit-identical in a 16-row tree pass and in a 1-row pass.
//
// Work split: one unit (CTA) per (row t, kv head g, segment of <= ATT_SEGSUB sub-chunks). Warp w
// stages the cached rows of sub-chunk w of the segment (coalesced cp.async into its own
// XOR-swizzled buffer). Two otherwise idle warps poll the words the QKV stage publishes, once per
// unit: warp ATT_WQ the 7 query rows of row t (into shared memory), warp ATT_WKV the pass rows
// (row t's ancestors) of the segment's K and V (into the staging buffers of the warps that hold
// their positions). After a named barrier each sub-chunk warp computes S = (q/8) K^T, the masked
// softmax and O = P V on the tensor cores (q as fp16 hi + lo A fragments, K and V B fragments by
// ldmatrix). Its record replaces its K rows in shared memory and the CTA combines the records. A
// row longer than one segment writes its records to global memory; the segment that arrives last
// combines them all.

constexpr int GQ = NQ / NKV;            // 7 query heads per KV head
constexpr int ATT_TICKETS = 1024;       // offset of the attention arrival counters in tickets
constexpr int ATT_REC = GQ * (2 + HD);  // records of a (row, kv head, sub-chunk): per head m, l, o[64]
constexpr int ATT_SEGSUB = 9;           // sub-chunks per unit (one per warp; shared-memory bound)
constexpr int ATT_WKV = 14;             // warp that polls the pass rows' K and V
constexpr int ATT_WQ = 15;              // warp that polls the query rows
static_assert(ATT_SEGSUB < ATT_WKV, "the polling warps hold no sub-chunk");

struct AttnSmem {
  // [warp][K, V][position][dim] staging; the warp's record overwrites its K rows once S is done
  alignas(128) __half kv[ATT_SEGSUB][2][ATT_SUB][HD];
  float q[GQ][HD];             // query rows of row t for the kv head's 7 heads
  int late;                    // a polling warp gave up (bounded wait)
  int last;
};
constexpr int ATT_REC_STRIDE = 2 * ATT_SUB * HD / 2;  // floats between the records of two warps
static_assert(ATT_REC * 4 <= ATT_SUB * HD * 2, "a record fits in the K rows of its buffer");

__device__ __forceinline__ int attn_subs(const RowInfo* ri, int t) {
  return (ri->pos + ri->depth[t] + 1 + ATT_SUB - 1) / ATT_SUB;
}
__device__ __forceinline__ int attn_segs(int nsub) { return (nsub + ATT_SEGSUB - 1) / ATT_SEGSUB; }

// Number of attention work units of a pass.
__device__ __forceinline__ int attn_units(const RowInfo* ri) {
  int total = 0;
  for (int t = 0; t < ri->n; ++t) total += NKV * attn_segs(attn_subs(ri, t));
  return total;
}

// Final output of (row t, kv head g) from its nsub records in sub-chunk order (record cc at
// base + cc * stride): M = max m_c, w_c = e^(m_c - M), O = sum_c o_c w_c / sum_c l_c w_c.
//
// The outputs go to the O projection as flagged words (two adjacent columns per word, written by
// the even lane), so that the O stage needs no grid barrier: GQ * HD = 448 outputs fill 14 warps
// exactly, so both lanes of a pair are always active.
__device__ __forceinline__ void attn_out(uint64_t* att_ll, uint32_t flag, int t, int col, float v) {
  const uint32_t u = __half_as_ushort(__float2half_rn(v));
  const uint32_t nb = __shfl_down_sync(0xffffffffu, u, 1);
  if ((col & 1) == 0) st_flagged(att_ll + act_index(t, col) / 2, u | (nb << 16), flag);
}
static_assert((GQ * HD) % 32 == 0, "attention outputs fill whole warps");

// Records in shared memory (one segment, nsub <= ATT_SEGSUB): every output thread forms the
// weights of its head itself (the same values in all 64 threads of the head), so no thread waits
// for another and the record loads and exponentials of all sub-chunks are in flight together.
__device__ __forceinline__ void attn_combine_local(uint64_t* att_ll, uint32_t flag, const float* base, int stride,
                                                   int nsub, int t, int g) {
  for (int i = threadIdx.x; i < GQ * HD; i += PASS_THREADS) {
    const int h = i / HD, d = i % HD;
    const float* rh = base + h * (2 + HD);
    float m[ATT_SEGSUB], l[ATT_SEGSUB], o[ATT_SEGSUB];
    float M = -INFINITY;
#pragma unroll
    for (int cc = 0; cc < ATT_SEGSUB; ++cc) {
      m[cc] = cc < nsub ? rh[cc * stride] : -INFINITY;
      l[cc] = cc < nsub ? rh[cc * stride + 1] : 0.f;
      o[cc] = cc < nsub ? rh[cc * stride + 2 + d] : 0.f;
      M = fmaxf(M, m[cc]);
    }
    float O = 0.f, Ls = 0.f;
#pragma unroll
    for (int cc = 0; cc < ATT_SEGSUB; ++cc) {
      if (cc < nsub) {
        const float w = expf(m[cc] - M);
        Ls = fmaf(l[cc], w, Ls);
        O = fmaf(o[cc], w, O);
      }
    }
    attn_out(att_ll, flag, t, (g * GQ + h) * HD + d, O / Ls);
  }
}

// Records in global memory (rows longer than one segment) hold up to max_subs records; their
// weights are recomputed per output (nsub can exceed the shared array).
__device__ __forceinline__ void attn_combine_global(const Scratch& s, const float* base, int stride, int nsub,
                                                    int t, int g) {
  for (int i = threadIdx.x; i < GQ * HD; i += PASS_THREADS) {
    const int h = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int cc = 0; cc < nsub; ++cc) M = fmaxf(M, __ldcg(base + cc * stride + h * (2 + HD)));
    float O = 0.f, Ls = 0.f;
    for (int cc = 0; cc < nsub; ++cc) {
      const float* r = base + cc * stride + h * (2 + HD);
      const float w = expf(__ldcg(r) - M);
      Ls = fmaf(__ldcg(r + 1), w, Ls);
      O = fmaf(__ldcg(r + 2 + d), w, O);
    }
    attn_out(s.att_ll, s.flag_q, t, (g * GQ + h) * HD + d, O / Ls);
  }
}

// fp16 hi + lo split of two values: hi = rn(v), lo = rn(v - hi).
__device__ __forceinline__ void split_half2(float a, float b, uint32_t& hi, uint32_t& lo) {
  const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
  hi = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
  const __half la = __float2half_rn(a - __half2float(ha)), lb = __float2half_rn(b - __half2float(hb));
  lo = (uint32_t)__half_as_ushort(la) | ((uint32_t)__half_as_ushort(lb) << 16);
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
// Byte offset of 16-byte chunk k (dims 8k..8k+7) of staged row r: XOR swizzle, so that the 8 rows
// of an 8x8 ldmatrix block fall in distinct bank groups.
__device__ __forceinline__ uint32_t kv_off(int r, int k) { return (uint32_t)(r * HD * 2 + ((k ^ (r & 7)) << 4)); }

// Barrier of the warps that take part in a unit: the nw sub-chunk warps and the two polling warps
// (named barrier 2; non-aligned form after a __syncwarp, as cons_sync).
__device__ __forceinline__ void attn_sync(int nw) {
  __syncwarp();
  asm volatile("barrier.sync 2, %0;" ::"r"((nw + 2) * 32) : "memory");
}

// Sub-chunk warp, first half: stage the cached rows of sub-chunk c (virtual positions 32c..32c+31)
// of row t: K rows then V rows (two cp.async groups, so S can start once K has landed). Lane copies
// 16-byte chunk (lane & 7) of rows (lane >> 3) + 4k, k < 8. Positions past the row are zeros; the
// pass's own rows (positions pos..L-1) are left to the polling warp.
__device__ __forceinline__ void attn_stage(const __half* kc, const __half* vc, const RowInfo* ri, int t, int c,
                                           __half* buf) {
  const int lane = threadIdx.x & 31;
  const int pos = ri->pos, L = pos + ri->depth[t] + 1;
  const uint64_t pol = policy_evict_last();
  const int ch = lane & 7;
  uint8_t* dk = reinterpret_cast<uint8_t*>(buf);
#pragma unroll
  for (int kv = 0; kv < 2; ++kv) {
    const __half* src = kv ? vc : kc;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int r = (lane >> 3) + 4 * k, jv = c * ATT_SUB + r;
      if (jv < pos || jv >= L)
        cp_async16(dk + kv * ATT_SUB * HD * 2 + kv_off(r, ch), src + (size_t)(jv < L ? jv : 0) * HD + ch * 8,
                   jv < L ? 16u : 0u, pol);
    }
    cp_async_commit();
  }
}

// Polling warp ATT_WQ: the 7 query rows (fp32) of row t for kv head g, as flagged words, into sm.q.
__device__ __noinline__ void attn_poll_q(const uint64_t* qw, uint32_t flag, AttnSmem& sm) {
  const int lane = threadIdx.x & 31;
  constexpr int PER = GQ * HD / 2 / 32;  // 16-byte loads (two words) per lane: 7
  uint32_t pend = (1u << PER) - 1u;
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 0; pend && it < (1u << 24); ++it) {
    // all loads of the round in flight before the first check (words 2u, 2u + 1, u = lane + 32k)
    uint64_t a[PER], b[PER];
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      a[k] = 0;
      b[k] = 0;
      if (pend >> k & 1u) ld_flagged2(qw + 2 * (lane + 32 * k), a[k], b[k]);
    }
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      if ((pend >> k & 1u) && (uint32_t)(a[k] >> 32) == flag && (uint32_t)(b[k] >> 32) == flag) {
        reinterpret_cast<float2*>(&sm.q[0][0])[lane + 32 * k] =
            make_float2(__uint_as_float((uint32_t)a[k]), __uint_as_float((uint32_t)b[k]));
        pend &= ~(1u << k);
      }
    }
    if ((it & 15) == 15 && globaltimer() - t0 > WAIT_NS) break;
  }
  if (pend) {
#pragma unroll
    for (int k = 0; k < PER; ++k)
      if (pend >> k & 1u) reinterpret_cast<float2*>(&sm.q[0][0])[lane + 32 * k] = make_float2(0.f, 0.f);
  }
  if (__any_sync(0xffffffffu, pend != 0) && lane == 0) sm.late = 1;
}

// Polling warp ATT_WKV: the pass rows among the segment's positions (row t's ancestors at virtual
// positions pos..L-1 in sub-chunks c0..c1-1), K and V from the flagged words of the QKV stage, into
// the staging buffers (sub-chunk c in buffer c - c0). Lane: 16-byte chunk (lane & 7) of rows.
__device__ __noinline__ void attn_poll_rows(const uint64_t* kw, const uint64_t* vw, uint32_t flag, const RowInfo* ri,
                                            int t, int c0, int c1, AttnSmem& sm) {
  const int lane = threadIdx.x & 31, ch = lane & 7;
  const int pos = ri->pos, L = pos + ri->depth[t] + 1;
  const int j0 = max(pos, c0 * ATT_SUB), j1 = min(L, c1 * ATT_SUB);  // positions to fill
  bool late = false;
  // at most 16 pass rows: lane handles rows (lane >> 3) + 4k of the range, k < 4, K and V
  uint32_t pend = 0;
#pragma unroll
  for (int k = 0; k < 4; ++k)
    if (j0 + (lane >> 3) + 4 * k < j1) pend |= 3u << (2 * k);
  const unsigned long long t0 = globaltimer();
  // source words of each (row, K / V) slot of this lane, fixed for the unit
  const uint64_t* src[8];
#pragma unroll
  for (int k = 0; k < 4; ++k)
#pragma unroll
    for (int kv = 0; kv < 2; ++kv) {
      const int jv = j0 + (lane >> 3) + 4 * k;
      const int prow = ri->path[t][min(max(jv - pos, 0), ROWS - 1)];
      src[2 * k + kv] = (kv ? vw : kw) + (size_t)prow * (HD / 2) + 4 * ch;
    }
  for (uint32_t it = 0; pend && it < (1u << 24); ++it) {
    // all loads of the round in flight before the first check
    uint64_t a[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      a[i][0] = a[i][1] = a[i][2] = a[i][3] = 0;
      if (pend >> i & 1u) {
        ld_flagged2(src[i], a[i][0], a[i][1]);
        ld_flagged2(src[i] + 2, a[i][2], a[i][3]);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int kv = 0; kv < 2; ++kv) {
        const int i = 2 * k + kv;
        if ((pend >> i & 1u) && (uint32_t)(a[i][0] >> 32) == flag && (uint32_t)(a[i][1] >> 32) == flag &&
            (uint32_t)(a[i][2] >> 32) == flag && (uint32_t)(a[i][3] >> 32) == flag) {
          const int jv = j0 + (lane >> 3) + 4 * k;
          const int c = jv / ATT_SUB, r = jv % ATT_SUB;
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(&sm.kv[c - c0][kv][0][0]) + kv_off(r, ch)) =
              make_uint4((uint32_t)a[i][0], (uint32_t)a[i][1], (uint32_t)a[i][2], (uint32_t)a[i][3]);
          pend &= ~(1u << i);
        }
      }
    if ((it & 15) == 15 && globaltimer() - t0 > WAIT_NS) break;
  }
  if (pend) {
    late = true;
#pragma unroll
    for (int k = 0; k < 4; ++k)
#pragma unroll
      for (int kv = 0; kv < 2; ++kv)
        if (pend >> (2 * k + kv) & 1u) {
          const int jv = j0 + (lane >> 3) + 4 * k, c = jv / ATT_SUB, r = jv % ATT_SUB;
          *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(&sm.kv[c - c0][kv][0][0]) + kv_off(r, ch)) =
              make_uint4(0u, 0u, 0u, 0u);
        }
  }
  if (__any_sync(0xffffffffu, late) && lane == 0) sm.late = 1;
}

// Sub-chunk warp, second half (after the unit's barrier): sub-chunk c of row t staged in buf (K
// rows then V rows), queries in sm.q. Writes the record to rec (the K rows of buf).
__device__ __noinline__ void attn_compute(const RowInfo* ri, int t, int c, const AttnSmem& sm, __half* buf,
                                          float* rec, unsigned long long* tr) {
#define ATT_DSTAMP(k, dep) do { if (tr) { const unsigned long long v_ = globaltimer_after(dep); if ((threadIdx.x & 31) == 0) tr[256 * (k)] = v_; } } while (0)
  const int lane = threadIdx.x & 31, gid = lane >> 2, t4 = lane & 3;
  const int L = ri->pos + ri->depth[t] + 1;
  // q * 0.125 (exact) as fp16 hi + lo A fragments of the 7 query heads: the hi halves in MMA rows
  // 0..6, the lo halves in rows 8..14 (rows 7 and 15 are zero), so that one MMA forms both
  // products and the two accumulator rows of a thread are added once at the end; dims
  // ks * 16 + 2 t4 + {0, 1} (a0 / a1) and + 8 (a2 / a3)
  uint32_t qa[4][2][2];  // [k-step][hi, lo][k 0..7, k 8..15]
  {
    const float* q = &sm.q[min(gid, GQ - 1)][0];
    const float z = gid < GQ ? ATTN_SCALE : 0.f;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const float2 x0 = *reinterpret_cast<const float2*>(q + ks * 16 + 2 * t4);
      const float2 x1 = *reinterpret_cast<const float2*>(q + ks * 16 + 8 + 2 * t4);
      split_half2(x0.x * z, x0.y * z, qa[ks][0][0], qa[ks][1][0]);
      split_half2(x1.x * z, x1.y * z, qa[ks][0][1], qa[ks][1][1]);
    }
  }
  ATT_DSTAMP(3, __uint_as_float(qa[3][1][1]));
  cp_async_wait<1>();  // the K rows (this lane's copies; __syncwarp makes the warp's visible)
  __syncwarp();
  const uint32_t sK = smem_u32(buf), sV = sK + ATT_SUB * HD * 2;
  ATT_DSTAMP(4, __uint_as_float(*reinterpret_cast<const uint32_t*>(buf)));
  const int mi = lane >> 3, ri8 = lane & 7;  // ldmatrix: this lane addresses row ri8 of block mi
  // S = q K^T: n-tile j = positions 8j..8j+7; one x4 load gives the B fragments of two k-steps.
  // sacc[j][e] is the hi product of position 8j + 2 t4 + e, sacc[j][2 + e] the lo product.
  float sacc[4][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int i = 0; i < 4; ++i) sacc[j][i] = 0.f;
    uint32_t kb[4][2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
      ldsm_x4(sK + kv_off(8 * j + ri8, 4 * hh + mi), kb[2 * hh][0], kb[2 * hh][1], kb[2 * hh + 1][0],
              kb[2 * hh + 1][1]);
#pragma unroll
    for (int ks = 0; ks < 4; ++ks)
      mma16816(sacc[j], qa[ks][0][0], qa[ks][1][0], qa[ks][0][1], qa[ks][1][1], kb[ks][0], kb[ks][1]);
#pragma unroll
    for (int e = 0; e < 2; ++e) sacc[j][e] += sacc[j][2 + e];
  }
  ATT_DSTAMP(5, sacc[3][0]);
  // masked softmax of query head gid over the 32 positions (position 8j + 2*t4 + e)
  const int cnt = L - c * ATT_SUB;
  float m = -INFINITY;
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sacc[j][e] = 8 * j + 2 * t4 + e < cnt ? sacc[j][e] : -INFINITY;
      m = fmaxf(m, sacc[j][e]);
    }
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
  m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
  float l = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      sacc[j][e] = expf(sacc[j][e] - m);
      l += sacc[j][e];
    }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  cp_async_wait<0>();  // the V rows
  __syncwarp();
  ATT_DSTAMP(6, __uint_as_float(*reinterpret_cast<const uint32_t*>(buf + ATT_SUB * HD)) + l);
  // P as the A operand: k-step kk = positions 16kk..16kk+15 = n-tiles 2kk (k 0..7) and 2kk+1
  // (k 8..15); hi halves in rows 0..6, lo halves in rows 8..14, as for q
  uint32_t pa[2][2][2];  // [kk][hi, lo][k 0..7, k 8..15]
#pragma unroll
  for (int kk = 0; kk < 2; ++kk) {
    split_half2(sacc[2 * kk][0], sacc[2 * kk][1], pa[kk][0][0], pa[kk][1][0]);
    split_half2(sacc[2 * kk + 1][0], sacc[2 * kk + 1][1], pa[kk][0][1], pa[kk][1][1]);
  }
  // O = P V: n-tile nd = dims 8nd..8nd+7; V B fragments by transposed ldmatrix, two n-tiles per x4.
  // The K rows are dead: the record goes there.
  float* r = rec + min(gid, GQ - 1) * (2 + HD);
#pragma unroll
  for (int np = 0; np < 4; ++np) {
    float oacc[2][4] = {};
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      uint32_t b00, b01, b10, b11;  // [n-tile 2np + x][b0, b1]
      ldsm_x4_trans(sV + kv_off(16 * kk + 8 * (mi & 1) + ri8, 2 * np + (mi >> 1)), b00, b01, b10, b11);
      mma16816(oacc[0], pa[kk][0][0], pa[kk][1][0], pa[kk][0][1], pa[kk][1][1], b00, b01);
      mma16816(oacc[1], pa[kk][0][0], pa[kk][1][0], pa[kk][0][1], pa[kk][1][1], b10, b11);
    }
    if (gid < GQ) {
#pragma unroll
      for (int x = 0; x < 2; ++x)
        *reinterpret_cast<float2*>(r + 2 + (2 * np + x) * 8 + 2 * t4) =
            make_float2(oacc[x][0] + oacc[x][2], oacc[x][1] + oacc[x][3]);
    }
    __syncwarp();
  }
  if (gid < GQ && t4 == 0) { r[0] = m; r[1] = l; }
  __syncwarp();
#undef ATT_DSTAMP
}

// One unit with PASS_THREADS threads: segment seg of (row t, kv head g).
// tr (performance tracing only): per-warp stamps at tr[256 * (8 * warp + step)]; the polling warps
// use steps 0 and 2 only, the unit-level stamps sit in warp 15's unused steps 5 and 7.
__device__ void attn_unit(const Scratch& s, int layer, int max_subs, int u, AttnSmem& sm,
                          unsigned long long* tr = nullptr) {
  const RowInfo* ri = s.ri;
  const int tid = threadIdx.x, warp = tid >> 5;
  int t = 0, rem = u, nsub = 1, nseg = 1;
  for (; t < ri->n; ++t) {
    nsub = attn_subs(ri, t);
    nseg = attn_segs(nsub);
    if (rem < NKV * nseg) break;
    rem -= NKV * nseg;
  }
  const int g = rem / nseg, seg = rem % nseg;
  const int c0 = seg * ATT_SEGSUB, c1 = min(nsub, c0 + ATT_SEGSUB), nw = c1 - c0;
  float* rec0 = reinterpret_cast<float*>(&sm.kv[0][0][0][0]);
  const size_t cache = (size_t)(layer * NKV + g) * s.max_ctx * HD;
  const size_t kvw = (size_t)ROWS * (HD / 2);
#define ATT_TSTAMP(k) do { if (tr && (tid & 31) == 0) tr[256 * (8 * warp + (k))] = globaltimer(); } while (0)
  if (tid == 0) sm.late = 0;
  cons_sync();
  ATT_TSTAMP(0);
  if (warp < nw) {
    attn_stage(s.kc + cache, s.vc + cache, ri, t, c0 + warp, &sm.kv[warp][0][0][0]);
    ATT_TSTAMP(1);
    attn_sync(nw);
  } else if (warp == ATT_WQ) {
    attn_poll_q(s.q_ll + t * H + g * GQ * HD, s.flag_q, sm);
    ATT_TSTAMP(2);
    attn_sync(nw);
  } else if (warp == ATT_WKV) {
    attn_poll_rows(s.kv_ll + g * kvw, s.kv_ll + (NKV + g) * kvw, s.flag_q, ri, t, c0, c1, sm);
    ATT_TSTAMP(2);
    attn_sync(nw);
  }
  if (warp < nw) {
    attn_compute(ri, t, c0 + warp, sm, &sm.kv[warp][0][0][0], rec0 + warp * ATT_REC_STRIDE,
                 tr ? tr + 256 * 8 * warp : nullptr);
    ATT_TSTAMP(7);
  }
  cons_sync();
  if (tid == 0 && sm.late) set_error(s.st, VP_DEV_ERR_TIMEOUT);
  if (tr && tid == 0) tr[256 * 125] = globaltimer();
#undef ATT_TSTAMP
  if (nseg == 1) {
    attn_combine_local(s.att_ll, s.flag_q, rec0, ATT_REC_STRIDE, nsub, t, g);
    cons_sync();
    if (tr && tid == 0) tr[256 * 127] = globaltimer();
    return;
  }
  float* base = s.att_part + (size_t)(t * NKV + g) * max_subs * ATT_REC;
  for (int i = tid; i < (c1 - c0) * ATT_REC; i += PASS_THREADS)
    base[(c0 + i / ATT_REC) * ATT_REC + i % ATT_REC] = rec0[(i / ATT_REC) * ATT_REC_STRIDE + i % ATT_REC];
  __threadfence();
  cons_sync();
  if (tid == 0) sm.last = atomicAdd(s.tickets + ATT_TICKETS + t * NKV + g, 1) == nseg - 1;
  cons_sync();
  if (sm.last) {
    __threadfence();
    attn_combine_global(s, base, ATT_REC, nsub, t, g);
    if (tid == 0) s.tickets[ATT_TICKETS + t * NKV + g] = 0;
  }
  cons_sync();
}

}  // namespace vp
