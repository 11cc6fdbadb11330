// The learned drafter on the device: proposes the next verify pass's draft tree from the request's
// committed tokens, between passes, so that the decode loop never returns to the host.
//
// Replaces the reference's k_ildraft (Sources/Engine/Shaders.swift:428-872), whose specification is
// tools/draft/ildraft.py (Drafter.features :519-692, the scorer :694-708, Drafter.tree :724-747).
// One CTA per request. For each context it expands (the committed tokens plus the path of a tree
// node) it finds the candidate next tokens and their 53 features, scores them with the table's MLP
// in float64, and keeps the 8 most probable; thread 0 grows the best-first tree from those.
//
// Data in device memory:
//  * the table (DraftTab): the sorted n-gram context keys with their counts and next tokens, the
//    copy rates (sorted by token or token pair), dense token flags and the MLP weights;
//  * the request (DraftReq, built on the host at request start: ildraft.py Drafter.begin): prompt
//    ids, their sorted distinct ids (copy candidates), the nearest training documents with their
//    sequences and sorted n-gram indexes, the association map.
// Every search is a binary search over sorted arrays; the per-context scans (the suffix of the
// output against the output itself and against the prompt) run over all threads.
#pragma once
#include "vp_common.cuh"

namespace vp {

constexpr int DR_THREADS = 256;
constexpr int DR_F = 53;               // features (ildraft.py FEATS)
constexpr int DR_H_MAX = 32;           // MLP hidden units supported
constexpr int DR_MAX_CAND = 1024;      // candidates of one context
constexpr int DR_MAX_NB = 16;          // nearest documents
constexpr int DR_MAXM_MAX = 16;        // longest suffix match supported
constexpr int DR_N_MAX = 8;            // highest n-gram order supported
constexpr int DR_HEAP = 8 + 16 * 8;    // best-first queue capacity (root + 15 expansions of 8)
constexpr int DR_VOCAB = 151936;
constexpr int DR_WORDS = (DR_VOCAB + 31) / 32;
constexpr int DR_SUMW = (DR_WORDS + 31) / 32;  // summary bitset: which words of a token bitset are set
static_assert(DR_SUMW <= DR_THREADS, "one thread per summary word");

// feature indices (ildraft.py FEATS order)
enum DrFeat {
  F_BIAS = 0, F_NG_P_LONG, F_NG_TOP_LONG, F_NG_ORD_LONG, F_NG_LCNT_LONG, F_NG_P_SUPP3, F_NG_P_SUPP10,
  F_NG_P1, F_NG_P2, F_NG_P3, F_NG_P4, F_NG_P5, F_NG_P6, F_NG_RANK2, F_NG_RANK3PLUS, F_NG_ENT_LOW,
  F_SF_M, F_SF_ANY, F_SF_M_GE3, F_PR_M, F_PR_ANY, F_PR_M_GE2, F_PR_FIRST,
  F_NB_SUM, F_NB_MSUM, F_NB_CNT, F_NB_MAXM, F_NB_TOP1, F_NB_TOP1_M,
  F_IS_STOP, F_IN_PROMPT, F_AGREE_NG_NB, F_AGREE_SF_NB,
  F_CP_PROP, F_CP_CTX1, F_CP_CTX2, F_CP_UNUSED, F_CP_FIRST_UNUSED, F_CP_SPACEVAR,
  F_ST_OPEN_FENCE, F_ST_OPEN_TICK, F_C_TICK, F_C_NL, F_ST_TICKS_ODD, F_ST_LEN, F_C_REPEAT,
  F_AS_MAX, F_AS_CNT, F_AS_CAND, F_ED_SUM, F_ED_CNT, F_ED_MAXM, F_ED_TOP1
};
static_assert(F_ED_TOP1 + 1 == DR_F, "53 features");

struct DrPair { uint32_t a, b; };       // (token, count) / (total, first << 3 | n)
struct DrRate { uint32_t tok; float v; };
struct DrRate2 { unsigned long long key; float v; uint32_t pad; };

struct DraftTab {
  const unsigned long long* ngky; const DrPair* ngvl; const DrPair* ngnx; int n_ng;
  const DrRate* prop; int n_prop;        // copy propensity, default 0.2
  const DrRate* cc1; int n_cc1;          // copy rate after a token, default 0.1
  const DrRate2* cc2; int n_cc2;         // copy rate after a token pair (t1 << 32 | t2), default 0.1
  const uint8_t* tflg;                   // [151936] bits 0-2 backticks, bit 3 newline
  const float* mlp;                      // W1[H][F], b1[H], W2[H], b2, WL[F]
  int N, MAXM, H, flags;
};

struct DraftReq {
  const int32_t* P; int np;              // prompt ids
  const int32_t* copy; int ncopy;        // sorted distinct prompt ids: copy candidates, prompt set
  const double* nb_score; int nnb;
  const int32_t* nb_seq_off;             // [nnb + 1] into nb_seq (TAIL + training output)
  const int32_t* nb_seq;
  const int32_t* nb_key_off;             // [nnb + 1] into nb_keys / nb_pos
  const unsigned long long* nb_keys;     // per document: sorted keys of its n-grams (1..MAXM)
  const int32_t* nb_pos;                 // index after the n-gram's first occurrence with a next token
  const int32_t* as_tok; const double* as_max; const int32_t* as_cnt; int nas;  // association map
  const int32_t* as_cand; int nascand;   // association candidates (sorted)
  const float* copy_prop;                // per copy id: its copy propensity (k_draft stages it), or null
  const double* copy_logit;              // and its feature log(p / (1 - p)) / 4, or null
};

struct DraftOut {
  int32_t* tree;        // VP_TREE_INTS: the next verify pass's tree
  int32_t* parents;     // optional [15]: node parents (-1 root), tokens, expansion top lists
  int32_t* tokens;
  int32_t* exp_tok;     // optional [16][8] top tokens of each expansion (-1: none)
  double* exp_p;        // [16][8] their probabilities
  int32_t* status;      // optional: 0 ok, bit 0 candidates capped, bit 1 a limit exceeded
};

__device__ __forceinline__ int dr_tail(int i) {
  return i == 0 ? 151645 : i == 1 ? 198 : i == 2 ? 151644 : i == 3 ? 77091 : 198;
}

template <typename T, typename K>
__device__ __forceinline__ int dr_find(const T* a, int n, K key, K (*get)(const T&)) {
  int lo = 0, hi = n;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (get(a[mid]) < key) lo = mid + 1; else hi = mid;
  }
  return (lo < n && get(a[lo]) == key) ? lo : -1;
}
__device__ __forceinline__ unsigned long long dr_u64(const unsigned long long& x) { return x; }
__device__ __forceinline__ uint32_t dr_rtok(const DrRate& x) { return x.tok; }
__device__ __forceinline__ unsigned long long dr_r2key(const DrRate2& x) { return x.key; }
__device__ __forceinline__ int dr_i32(const int32_t& x) { return x; }

// Staging caps: the committed output, the prompt and the distinct prompt ids (with their copy
// propensities) are copied into shared memory once per launch when they fit, so the per-context
// scans and searches run on shared memory; longer requests read them from global memory.
constexpr int DR_OUT_CAP = 2048;
constexpr int DR_PROMPT_CAP = 2048;
constexpr int DR_COPY_CAP = 2048;
constexpr int DR_AS_CAP = 1024;           // association map and candidates
constexpr int DR_SMALL = 96;   // (token, bits) of the small sources: n-gram lists, self, first prompt match, votes

struct DrShared {
  uint32_t used[DR_WORDS];                 // bitset of the committed output's tokens
  uint32_t mark[DR_WORDS];                 // candidate tokens of the current context
  uint32_t msum[DR_SUMW];                  // its nonzero words
  uint32_t prm[DR_WORDS];                  // tokens after a longest prompt match (source DS_PR)
  int ctok[DR_MAX_CAND];                   // the context's distinct candidates, ascending
  uint32_t cbits[DR_MAX_CAND];             // their source bits
  double prob[DR_MAX_CAND];
  unsigned long long small[DR_SMALL];      // (token << 32) | bits of the small sources
  int nsmall;
  int outs[DR_OUT_CAP];                    // staged copies (see the caps above)
  int prs[DR_PROMPT_CAP];
  int cps[DR_COPY_CAP];
  float cpp[DR_COPY_CAP];                  // copy propensity (NaN: not in the table)
  double cplg[DR_COPY_CAP];                // its feature, log(p / (1 - p)) / 4
  int ast[DR_AS_CAP], ascn[DR_AS_CAP], asc[DR_AS_CAP];
  double asmx[DR_AS_CAP];
  double nbs[DR_MAX_NB];
  double mlpd[DR_H_MAX * DR_F + 2 * DR_H_MAX + 1 + DR_F];  // W1, b1, W2, b2, WL as float64
  DrPair ngtop[DR_N_MAX + 1][8];           // the context's n-gram next-token lists
  int nbhit[DR_MAX_NB][DR_MAXM_MAX + 1];   // per document and suffix length: next token or -1
  unsigned long long hsh[DR_MAXM_MAX + 1]; // key of the context's last n tokens
  int dist_tot[DR_N_MAX + 1], dist_first[DR_N_MAX + 1], dist_n[DR_N_MAX + 1];
  int long_n, supp3, supp10, top_long, ent_low;
  int vote_tok[DR_MAX_NB], vote_n[DR_MAX_NB];
  int path[16], npath;
  int ncand, red_i[DR_THREADS / 32];
  double red_d[DR_THREADS / 32];
  int self_n, self_tok, pr_n, pr_first_e, first_unused, ticks0, capped;
  double c1, c2;
  unsigned long long wtop_k[DR_THREADS / 32][8];  // per-warp top 8 (key, candidate index)
  int wtop_i[DR_THREADS / 32][8];
  // best-first queue and the tree
  double hk[DR_HEAP]; int hseq[DR_HEAP], hpar[DR_HEAP], htok[DR_HEAP], hn, hctr;
  int npar[16], ntok[16], nodes, cur, go;
  int top_tok[8]; double top_p[8];
#ifdef VP_DRAFT_TRACE
  unsigned long long tacc[32], tlast;  // per-phase time summed over the expansions (thread 0)
#endif
};

#ifdef VP_DRAFT_TRACE
__device__ unsigned long long g_dr_trace[32];
#define DR_T(sh, k)                                       \
  do {                                                    \
    if (threadIdx.x == 0) {                               \
      const unsigned long long t_ = globaltimer();        \
      (sh).tacc[k] += t_ - (sh).tlast;                    \
      (sh).tlast = t_;                                    \
    }                                                     \
  } while (0)
#else
#define DR_T(sh, k) do { } while (0)
#endif

// source bits of a candidate
constexpr uint32_t DS_NG = 1, DS_SELF = 2, DS_PR = 4, DS_PRFIRST = 8, DS_NB = 16, DS_COPY = 32, DS_ASC = 64;

struct DrCtx {  // the context being expanded: TAIL + out0 + path
  const int32_t* out0; int lo0;
  const int* path; int np;
  __device__ __forceinline__ int lo() const { return lo0 + np; }
  __device__ __forceinline__ int out(int i) const { return i < lo0 ? out0[i] : path[i - lo0]; }
  __device__ __forceinline__ int ctx(int i) const { return i < 5 ? dr_tail(i) : out(i - 5); }
  __device__ __forceinline__ int L() const { return 5 + lo(); }
};

// Warp reductions through redux.sync (one instruction per 32-bit word) instead of shuffle trees.
__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
  const unsigned hi = (unsigned)(v >> 32);
  const unsigned mhi = __reduce_max_sync(0xffffffffu, hi);
  const unsigned mlo = __reduce_max_sync(0xffffffffu, hi == mhi ? (unsigned)v : 0u);
  return ((unsigned long long)mhi << 32) | mlo;
}
// The lane holding the largest key (ties: the lowest idx; idx -1 = none, and key 0 marks an empty
// lane): key and idx of the winner in every lane.
__device__ __forceinline__ void warp_argmax(unsigned long long& key, int& idx) {
  const unsigned long long m = warp_max_u64(key);
  idx = (int)__reduce_min_sync(0xffffffffu, key == m ? (unsigned)idx : 0xffffffffu);
  key = m;
}
// Doubles as unsigned integers of the same order (for max / min through integer reductions).
__device__ __forceinline__ unsigned long long dr_ord(double d) {
  const unsigned long long u = (unsigned long long)__double_as_longlong(d);
  return (u >> 63) ? ~u : (u | 0x8000000000000000ull);
}
__device__ __forceinline__ double dr_unord(unsigned long long u) {
  return __longlong_as_double((long long)((u >> 63) ? (u & 0x7fffffffffffffffull) : ~u));
}

// Block reductions (256 threads) with a fixed combination order.
__device__ __forceinline__ int dr_max_i(int v, DrShared& sh) {
  v = __reduce_max_sync(0xffffffffu, v);
  if ((threadIdx.x & 31) == 0) sh.red_i[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = sh.red_i[0];
  for (int w = 1; w < DR_THREADS / 32; ++w) r = max(r, sh.red_i[w]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ int dr_min_i(int v, DrShared& sh) { return -dr_max_i(-v, sh); }
__device__ __forceinline__ double dr_max_d(double v, DrShared& sh) {
  const unsigned long long u = warp_max_u64(dr_ord(v));
  if ((threadIdx.x & 31) == 0) sh.red_d[threadIdx.x >> 5] = dr_unord(u);
  __syncthreads();
  double r = sh.red_d[0];
  for (int w = 1; w < DR_THREADS / 32; ++w) r = fmax(r, sh.red_d[w]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ double dr_sum_d(double v, DrShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  if ((threadIdx.x & 31) == 0) sh.red_d[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = sh.red_d[0];
  for (int w = 1; w < DR_THREADS / 32; ++w) r += sh.red_d[w];
  __syncthreads();
  return r;
}

__device__ __forceinline__ bool dr_used(const DrShared& sh, const DrCtx& c, int tok) {
  if (tok >= 0 && tok < DR_VOCAB && (sh.used[tok >> 5] >> (tok & 31) & 1u)) return true;
  for (int i = 0; i < c.np; ++i)
    if (c.path[i] == tok) return true;
  return false;
}
__device__ __forceinline__ uint8_t dr_flag(const DraftTab& T, int tok) {
  return (tok >= 0 && tok < DR_VOCAB) ? T.tflg[tok] : 0;
}
__device__ __forceinline__ double dr_prop(const DraftTab& T, int tok, double dflt) {
  const int i = dr_find(T.prop, T.n_prop, (uint32_t)tok, dr_rtok);
  return i >= 0 ? (double)T.prop[i].v : dflt;
}
// Copy propensity (default 0.2) of the copy id at index i of R.copy: from the staged per-id table
// when there is one (NaN there: not in the table).
__device__ __forceinline__ double dr_copy_prop(const DraftTab& T, const DraftReq& R, int i, int tok) {
  if (R.copy_prop) {
    const float v = R.copy_prop[i];
    return v == v ? (double)v : 0.2;
  }
  return dr_prop(T, tok, 0.2);
}
// Copy propensity of a prompt id.
__device__ __forceinline__ double dr_prompt_prop(const DraftTab& T, const DraftReq& R, int tok) {
  if (R.copy_prop) {
    const int i = dr_find(R.copy, R.ncopy, tok, dr_i32);
    if (i >= 0) return dr_copy_prop(T, R, i, tok);
  }
  return dr_prop(T, tok, 0.2);
}
// A candidate token: marked in the context's set (duplicates merge for free).
__device__ __forceinline__ void dr_mark(DrShared& sh, int tok) {
  if (tok < 0 || tok >= DR_VOCAB) return;
  atomicOr(&sh.mark[tok >> 5], 1u << (tok & 31));
  atomicOr(&sh.msum[tok >> 10], 1u << ((tok >> 5) & 31));
}
// A candidate from a small source, whose bits are merged after the compaction.
__device__ __forceinline__ void dr_push_small(DrShared& sh, int tok, uint32_t bits) {
  if (tok < 0 || tok >= DR_VOCAB) return;
  dr_mark(sh, tok);
  const int k = atomicAdd(&sh.nsmall, 1);
  if (k < DR_SMALL) sh.small[k] = ((unsigned long long)(uint32_t)tok << 32) | bits;
}

// Longest common suffix of seq[0..e) and the output (both end-aligned), at most cap.
template <typename Seq>
__device__ __forceinline__ int dr_suffix(const Seq& s, int e, const DrCtx& c, int cap) {
  const int lo = c.lo();
  int k = 0;
  while (k < cap && k < e && s(e - 1 - k) == c.out(lo - 1 - k)) ++k;
  return k;
}

// acc[j] += W[(h + j) * DR_F + f] * x[f] for the features f in [F0, F1), in feature order.
template <int F0, int F1, int J>
__device__ __forceinline__ void dr_dot(const double* W, int h, const double (&x)[DR_F], double (&acc)[J]) {
#pragma unroll
  for (int f = F0; f < F1; ++f)
#pragma unroll
    for (int j = 0; j < J; ++j) acc[j] = fma(W[(h + j) * DR_F + f], x[f], acc[j]);
}
// The same over every feature group that can be nonzero (see the MLP in dr_expand).
template <int J>
__device__ __forceinline__ void dr_dot_groups(const double* W, int h, const double (&x)[DR_F], double (&acc)[J],
                                              bool has_nb, bool has_as) {
  dr_dot<0, F_NB_SUM, J>(W, h, x, acc);
  if (has_nb) dr_dot<F_NB_SUM, F_IS_STOP, J>(W, h, x, acc);
  dr_dot<F_IS_STOP, F_AGREE_NG_NB, J>(W, h, x, acc);
  if (has_nb) dr_dot<F_AGREE_NG_NB, F_CP_PROP, J>(W, h, x, acc);
  dr_dot<F_CP_PROP, F_AS_MAX, J>(W, h, x, acc);
  if (has_as) dr_dot<F_AS_MAX, F_ED_SUM, J>(W, h, x, acc);
}
static_assert(F_NB_SUM < F_IS_STOP && F_IS_STOP < F_AGREE_NG_NB && F_AGREE_NG_NB < F_CP_PROP &&
              F_CP_PROP < F_AS_MAX && F_AS_MAX < F_ED_SUM && F_ED_SUM + 4 == DR_F, "feature groups in order");

// Candidates and probabilities of the next token after the context; leaves the top ntop (<= 8;
// probability descending, token ascending) in sh.top_tok / top_p (-1: fewer candidates or past
// ntop).
//
// The candidate set is a bitset over the vocabulary (duplicates from several sources merge by
// themselves), compacted in ascending token order by a block scan; the source bits of the large
// sources (prompt matches, copy ids, association candidates) are set membership tests, those of the
// small ones (n-gram lists, self match, first prompt match, votes) are merged after the compaction.
__device__ void dr_expand(const DraftTab& T, const DraftReq& R, const DrCtx& c, DrShared& sh, int ntop) {
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int L = c.L(), lo = c.lo();
  const int nmax = max(T.N, T.MAXM);
  DR_T(sh, 0);
  // keys of the context's last n tokens: FNV-1a 64 over the order byte, then the tokens (u32 LE)
  if (tid >= 1 && tid <= nmax && tid <= L) {
    unsigned long long h = 0xcbf29ce484222325ull;
    h = (h ^ (unsigned long long)tid) * 0x100000001b3ull;
    for (int i = L - tid; i < L; ++i) {
      const uint32_t t = (uint32_t)c.ctx(i);
#pragma unroll
      for (int b = 0; b < 4; ++b) h = (h ^ (unsigned long long)((t >> (8 * b)) & 0xffu)) * 0x100000001b3ull;
    }
    sh.hsh[tid] = h;
  }
  if (tid == 0) { sh.self_n = 0; sh.pr_n = 0; sh.nsmall = 0; }
  __syncthreads();
  DR_T(sh, 1);
  // the table searches, one work item each: n-gram distributions of orders 1..N (their next-token
  // lists staged), the copy rates after the last token and after the last pair, and every
  // (neighbour document, suffix length) key
  const int mm = min(T.MAXM, L);
  const int n_items = T.N + 2 + R.nnb * mm;
  for (int w = tid; w < n_items; w += DR_THREADS) {
    if (w < T.N) {
      const int n = w + 1;
      int tot = -1, first = 0, cnt = 0;
      if (n <= L) {
        const int i = dr_find(T.ngky, T.n_ng, sh.hsh[n], dr_u64);
        if (i >= 0) { tot = (int)T.ngvl[i].a; first = (int)(T.ngvl[i].b >> 3); cnt = (int)(T.ngvl[i].b & 7u); }
      }
      sh.dist_tot[n] = tot; sh.dist_first[n] = first; sh.dist_n[n] = cnt;
      for (int i = 0; i < cnt; ++i) sh.ngtop[n][i] = T.ngnx[first + i];
    } else if (w == T.N) {
      const int i1 = dr_find(T.cc1, T.n_cc1, (uint32_t)c.ctx(L - 1), dr_rtok);
      sh.c1 = i1 >= 0 ? (double)T.cc1[i1].v : 0.1;
    } else if (w == T.N + 1) {
      const unsigned long long k2 = ((unsigned long long)(uint32_t)c.ctx(L - 2) << 32) | (uint32_t)c.ctx(L - 1);
      const int i2 = dr_find(T.cc2, T.n_cc2, k2, dr_r2key);
      sh.c2 = i2 >= 0 ? (double)T.cc2[i2].v : 0.1;
    } else {
      const int r = (w - T.N - 2) / mm, n = 1 + (w - T.N - 2) % mm;
      const int k0 = R.nb_key_off[r], k1 = R.nb_key_off[r + 1];
      const int i = dr_find(R.nb_keys + k0, k1 - k0, sh.hsh[n], dr_u64);
      sh.nbhit[r][n] = i >= 0 ? R.nb_seq[R.nb_seq_off[r] + R.nb_pos[k0 + i]] : -1;
    }
  }
  __syncthreads();
  // each neighbour's vote: the next token after the longest context suffix found in it
  if (tid < R.nnb) {
    int tok = -1, got = 0;
    for (int n = mm; n >= 1; --n)
      if (sh.nbhit[tid][n] >= 0) { tok = sh.nbhit[tid][n]; got = n; break; }
    sh.vote_tok[tid] = tok; sh.vote_n[tid] = got;
  }
  DR_T(sh, 2);
  // self lookup: the longest suffix of the output found earlier in it (k(e) for next index e), the
  // latest such occurrence
  int best = 0;
  const int capo = min(T.MAXM, lo - 1);
  for (int e = 1 + tid; e <= lo - 1; e += DR_THREADS) best = max(best, dr_suffix([&](int i) { return c.out(i); }, e, c, capo));
  const int self_n = dr_max_i(best, sh);
  if (self_n > 0) {
    int last = -1;
    for (int e = 1 + tid; e <= lo - 1; e += DR_THREADS)
      if (dr_suffix([&](int i) { return c.out(i); }, e, c, capo) >= self_n) last = max(last, e);
    const int e = dr_max_i(last, sh);
    if (tid == 0) { sh.self_n = self_n; sh.self_tok = c.out(e); }
  }
  DR_T(sh, 3);
  // prompt lookup: every occurrence of the longest suffix of the output found in the prompt
  best = 0;
  const int capp = min(T.MAXM, lo);
  for (int e = 1 + tid; e <= R.np - 1; e += DR_THREADS)
    best = max(best, dr_suffix([&](int i) { return R.P[i]; }, e, c, capp));
  const int pr_n = dr_max_i(best, sh);
  if (tid == 0) sh.pr_n = pr_n;
  DR_T(sh, 4);
  // the candidates
  if (pr_n > 0) {
    int first = 0x7fffffff;
    for (int e = 1 + tid; e <= R.np - 1; e += DR_THREADS)
      if (dr_suffix([&](int i) { return R.P[i]; }, e, c, capp) >= pr_n) {
        const int t = R.P[e];
        if (t >= 0 && t < DR_VOCAB) atomicOr(&sh.prm[t >> 5], 1u << (t & 31));
        dr_mark(sh, t);
        first = min(first, e);
      }
    first = dr_min_i(first, sh);
    if (tid == 0) { sh.pr_first_e = first; dr_push_small(sh, R.P[first], DS_PRFIRST); }
  }
  if (tid >= 1 && tid <= T.N && sh.dist_tot[tid] >= 0)
    for (int i = 0; i < sh.dist_n[tid]; ++i) dr_push_small(sh, (int)sh.ngtop[tid][i].a, DS_NG);
  if (tid == 0) {
    int ln = 0, s3 = 0, s10 = 0;
    for (int n = 1; n <= T.N; ++n)
      if (sh.dist_tot[n] >= 0) {
        ln = n;
        if (sh.dist_tot[n] >= 3) s3 = n;
        if (sh.dist_tot[n] >= 10) s10 = n;
      }
    sh.long_n = ln; sh.supp3 = s3; sh.supp10 = s10;
    sh.top_long = -1; sh.ent_low = 0;
    if (ln) {
      const DrPair* top = sh.ngtop[ln];
      sh.top_long = sh.dist_n[ln] > 0 ? (int)top[0].a : -1;
      double ent = 0.0;
      const double tot = (double)sh.dist_tot[ln];
      for (int i = 0; i < sh.dist_n[ln]; ++i) {
        const double q = (double)top[i].b / tot;
        ent = ent + q * log(q);
      }
      sh.ent_low = -ent < 0.3;
    }
    if (sh.self_n > 0) dr_push_small(sh, sh.self_tok, DS_SELF);
  }
  if (tid < R.nnb && sh.vote_tok[tid] >= 0) dr_push_small(sh, sh.vote_tok[tid], DS_NB);
  DR_T(sh, 5);
  // the first prompt id not in the output whose copy propensity exceeds 0.3
  {
    int fu = 0x7fffffff;
    for (int j = tid; j < R.np; j += DR_THREADS)
      if (!dr_used(sh, c, R.P[j]) && dr_prompt_prop(T, R, R.P[j]) > 0.3) fu = min(fu, j);
    fu = dr_min_i(fu, sh);
    if (tid == 0) sh.first_unused = fu < R.np ? R.P[fu] : -1;
  }
  for (int j = tid; j < R.ncopy; j += DR_THREADS) dr_mark(sh, R.copy[j]);
  for (int j = tid; j < R.nascand; j += DR_THREADS) dr_mark(sh, R.as_cand[j]);
  __syncthreads();
  DR_T(sh, 6);
  // the distinct candidates in ascending token order: thread t takes the set words of summary word
  // t (32 words of the bitset), counts their marks, a block scan gives its first index, it writes
  // its tokens (and the prompt-match bit) and clears its words for the next context
  const uint32_t sw = tid < DR_SUMW ? sh.msum[tid] : 0u;
  int cnt = 0;
  for (uint32_t m = sw; m; m &= m - 1) cnt += __popc(sh.mark[tid * 32 + __ffs(m) - 1]);
  int incl = cnt;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) sh.red_i[wid] = incl;
  __syncthreads();
  int idx = incl - cnt, total = 0;
  for (int w = 0; w < DR_THREADS / 32; ++w) {
    if (w < wid) idx += sh.red_i[w];
    total += sh.red_i[w];
  }
  for (uint32_t sm_ = sw; sm_; sm_ &= sm_ - 1) {
    const int w = tid * 32 + __ffs(sm_) - 1;
    uint32_t m = sh.mark[w];
    const uint32_t pm = sh.prm[w];
    while (m) {
      const int b = __ffs(m) - 1;
      if (idx < DR_MAX_CAND) {
        sh.ctok[idx] = w * 32 + b;
        sh.cbits[idx] = (pm >> b & 1u) ? DS_PR : 0u;
      }
      ++idx;
      m &= m - 1;
    }
    sh.mark[w] = 0u;
    sh.prm[w] = 0u;
  }
  if (tid < DR_SUMW) sh.msum[tid] = 0u;
  const int nc = min(total, DR_MAX_CAND);  // past the cap: the lowest token ids are kept
  if (tid == 0 && total > DR_MAX_CAND) sh.capped = 1;
  __syncthreads();
  for (int k = tid; k < min(sh.nsmall, DR_SMALL); k += DR_THREADS) {
    const int i = dr_find(sh.ctok, nc, (int)(sh.small[k] >> 32), dr_i32);
    if (i >= 0) atomicOr(&sh.cbits[i], (uint32_t)sh.small[k]);
  }
  __syncthreads();
  DR_T(sh, 7);
  // features and scores, one candidate per thread, float64 (ildraft.py:519-701)
  const double ticks_odd = (double)((sh.ticks0 + [&] {
    int t = 0;
    for (int i = 0; i < c.np; ++i) t += dr_flag(T, c.path[i]) & 7;
    return t;
  }()) % 2);
  const int out_first = lo > 0 ? c.out(0) : -1;
  const double open_fence = (out_first == 73594 || out_first == 13874) ? 1.0 : 0.0;
  const double open_tick = out_first == 63 ? 1.0 : 0.0;
  const double st_len = (double)min(lo, 32) / 32.0;
  const bool has_nb = R.nnb > 0, has_as = R.nas > 0 || R.nascand > 0;
  const double* W1 = sh.mlpd;
  const double* b1 = W1 + T.H * DR_F;
  const double* W2 = b1 + T.H;
  const double b2 = W2[T.H];
  const double* WL = W2 + T.H + 1;
  for (int ci = tid; ci < nc; ci += DR_THREADS) {
    const int tok = sh.ctok[ci];
    const int icopy = dr_find(R.copy, R.ncopy, tok, dr_i32);
    const bool in_p = icopy >= 0;
    const bool in_as = R.nascand > 0 && dr_find(R.as_cand, R.nascand, tok, dr_i32) >= 0;
    const uint32_t src = sh.cbits[ci] | (in_p ? DS_COPY : 0u) | (in_as ? DS_ASC : 0u);
    double x[DR_F];
#pragma unroll
    for (int f = 0; f < DR_F; ++f) x[f] = 0.0;
    x[F_BIAS] = 1.0;
    // (unrolled over the orders, so that every index of x is a constant and x stays in registers)
#pragma unroll
    for (int n = 1; n <= DR_N_MAX; ++n) {
      if (n > T.N || sh.dist_tot[n] < 0) continue;
      const DrPair* top = sh.ngtop[n];
      int cnt_n = 0, rank = -1;
      for (int i = 0; i < sh.dist_n[n]; ++i)
        if ((int)top[i].a == tok) { cnt_n = (int)top[i].b; rank = i; break; }
      if (n == sh.long_n && rank == 1) x[F_NG_RANK2] = 1.0;
      if (n == sh.long_n && rank >= 2) x[F_NG_RANK3PLUS] = 1.0;
      if (cnt_n) {
        const double p = (double)cnt_n / (double)sh.dist_tot[n];
        if (n <= 6) x[F_NG_P1 + (n <= 6 ? n - 1 : 0)] = p;
        if (n == sh.long_n) {
          x[F_NG_P_LONG] = p;
          x[F_NG_ORD_LONG] = (double)n / 6.0 * p;
          x[F_NG_LCNT_LONG] = log1p((double)cnt_n);
        }
        if (n == sh.supp3) x[F_NG_P_SUPP3] = p;
        if (n == sh.supp10) x[F_NG_P_SUPP10] = p;
      }
    }
    if (tok == sh.top_long) {
      x[F_NG_TOP_LONG] = 1.0;
      if (sh.ent_low) x[F_NG_ENT_LOW] = 1.0;
    }
    if (src & DS_SELF) {
      x[F_SF_M] = (double)sh.self_n / 4.0;
      x[F_SF_ANY] = 1.0;
      x[F_SF_M_GE3] = sh.self_n >= 3 ? 1.0 : 0.0;
    }
    if (src & DS_PR) {
      x[F_PR_M] = (double)sh.pr_n / 4.0;
      x[F_PR_ANY] = 1.0;
      x[F_PR_M_GE2] = sh.pr_n >= 2 ? 1.0 : 0.0;
      if (src & DS_PRFIRST) x[F_PR_FIRST] = 1.0;
    }
    if (src & DS_NB) {
      double s1 = 0.0, s2 = 0.0;
      int cv = 0, mx = 0;
      for (int r = 0; r < R.nnb; ++r)
        if (sh.vote_tok[r] == tok) {
          const int m8 = min(sh.vote_n[r], 8);
          s1 = s1 + R.nb_score[r];
          s2 = s2 + R.nb_score[r] * (double)m8 / 8.0;
          ++cv;
          mx = max(mx, m8);
          if (r == 0) { x[F_NB_TOP1] = 1.0; x[F_NB_TOP1_M] = (double)m8 / 8.0; }
        }
      x[F_NB_SUM] = s1;
      x[F_NB_MSUM] = s2;
      x[F_NB_CNT] = (double)cv / (double)max(1, R.nnb);
      x[F_NB_MAXM] = (double)mx / 8.0;
    }
    const bool used = dr_used(sh, c, tok);
    if (src & DS_COPY) {
      if (R.copy_logit) {
        x[F_CP_PROP] = R.copy_logit[icopy];
      } else {
        const double pt = dr_copy_prop(T, R, icopy, tok);
        x[F_CP_PROP] = log(pt / (1.0 - pt)) / 4.0;
      }
      x[F_CP_CTX1] = sh.c1;
      x[F_CP_CTX2] = sh.c2;
      x[F_CP_UNUSED] = used ? 0.0 : 1.0;
      x[F_CP_FIRST_UNUSED] = tok == sh.first_unused ? 1.0 : 0.0;
      x[F_CP_SPACEVAR] = 0.0;
    }
    if (src & DS_ASC) x[F_AS_CAND] = 1.0;
    x[F_IS_STOP] = (tok == 151645 || tok == 151643) ? 1.0 : 0.0;
    x[F_IN_PROMPT] = in_p ? 1.0 : 0.0;
    x[F_AGREE_NG_NB] = x[F_NG_TOP_LONG] * fmin(1.0, 2.0 * x[F_NB_CNT]);
    x[F_AGREE_SF_NB] = x[F_SF_ANY] * fmin(1.0, 2.0 * x[F_NB_CNT]);
    const uint8_t fl = dr_flag(T, tok);
    x[F_ST_OPEN_FENCE] = open_fence;
    x[F_ST_OPEN_TICK] = open_tick;
    x[F_C_TICK] = (fl & 7) ? 1.0 : 0.0;
    x[F_C_NL] = (fl & 8) ? 1.0 : 0.0;
    x[F_ST_TICKS_ODD] = ticks_odd;
    x[F_ST_LEN] = st_len;
    x[F_C_REPEAT] = used ? 1.0 : 0.0;
    const int ai = dr_find(R.as_tok, R.nas, tok, dr_i32);
    if (ai >= 0) {
      x[F_AS_MAX] = R.as_max[ai] / 4.0;
      x[F_AS_CNT] = (double)min(R.as_cnt[ai], 4) / 4.0;
    }
    DR_T(sh, 11);
    // score = W2 . relu(W1 x + b1) + b2 + WL . x; eight hidden units at a time (each one its own
    // chain in feature order, the units summed in order). Feature groups that are zero for every
    // candidate of the request are left out of the chains (a zero term leaves an fma chain's value
    // unchanged): the neighbour votes and their agreements without neighbours, the association
    // features without an association map, and the edited-neighbour features always (they need the
    // tokenizer, which this build does not have, so they are zero as in the oracle).
    double s = 0.0;
    int h = 0;
    for (; h + 8 <= T.H; h += 8) {
      double a[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] = 0.0;
      dr_dot_groups<8>(W1, h, x, a, has_nb, has_as);
#pragma unroll
      for (int j = 0; j < 8; ++j) s = fma(W2[h + j], fmax(a[j] + b1[h + j], 0.0), s);
    }
    for (; h < T.H; ++h) {
      double a[1] = {0.0};
      dr_dot_groups<1>(W1, h, x, a, has_nb, has_as);
      s = fma(W2[h], fmax(a[0] + b1[h], 0.0), s);
    }
    double lin[1] = {0.0};
    dr_dot_groups<1>(WL, 0, x, lin, has_nb, has_as);
    sh.prob[ci] = s + b2 + lin[0];
    DR_T(sh, 13);
  }
  __syncthreads();
  DR_T(sh, 8);
  // softmax with a null option of score 0
  double m = -INFINITY;
  for (int ci = tid; ci < nc; ci += DR_THREADS) m = fmax(m, sh.prob[ci]);
  m = fmax(dr_max_d(m, sh), 0.0);
  double z = 0.0;
  for (int ci = tid; ci < nc; ci += DR_THREADS) z += exp(sh.prob[ci] - m);
  z = dr_sum_d(z, sh) + exp(-m);
  for (int ci = tid; ci < nc; ci += DR_THREADS) sh.prob[ci] = exp(sh.prob[ci] - m) / z;
  __syncthreads();
  DR_T(sh, 9);
  // the 8 most probable, probability descending then token (= index) ascending: each warp picks
  // the 8 best of its candidates, then warp 0 the 8 best of those 64. A probability's key is its
  // bit pattern plus one (monotonic for non-negative doubles); 0 marks none (taken entries hold
  // -2.0, which is not a probability).
#pragma unroll 1
  for (int k = 0; k < ntop; ++k) {
    unsigned long long bk = 0;
    int bi = -1;
    for (int ci = tid; ci < nc; ci += DR_THREADS) {
      const long long kb = __double_as_longlong(sh.prob[ci]);
      if (kb >= 0 && (unsigned long long)kb + 1 > bk) { bk = (unsigned long long)kb + 1; bi = ci; }
    }
    warp_argmax(bk, bi);
    if (lane == 0) {
      sh.wtop_k[wid][k] = bk;
      sh.wtop_i[wid][k] = bi;
      if (bi >= 0) sh.prob[bi] = -2.0;  // taken
    }
    __syncwarp();
  }
  DR_T(sh, 14);
  __syncthreads();
  DR_T(sh, 15);
  if (wid == 0) {
    constexpr int NW = DR_THREADS / 32;  // 8 warps x 8 entries: two per lane
    const bool used_k = (lane & 7) < ntop;  // entries past ntop were not filled
    unsigned long long k0 = used_k ? sh.wtop_k[lane >> 3][lane & 7] : 0ull;
    unsigned long long k1 = used_k ? sh.wtop_k[(NW / 2) + (lane >> 3)][lane & 7] : 0ull;
    int i0 = used_k ? sh.wtop_i[lane >> 3][lane & 7] : -1, i1 = used_k ? sh.wtop_i[(NW / 2) + (lane >> 3)][lane & 7] : -1;
    if (lane < 8) {
      sh.top_tok[lane] = -1;
      sh.top_p[lane] = 0.0;
    }
    __syncwarp();
#pragma unroll 1
    for (int k = 0; k < ntop; ++k) {
#ifdef VP_DRAFT_TRACE
      if (tid == 0) sh.tacc[16 + k] = clock64();
#endif
      unsigned long long bk = k0;
      int bi = i0;
      if (k1 > bk || (k1 == bk && k1 != 0 && i1 < bi)) { bk = k1; bi = i1; }
      warp_argmax(bk, bi);
      if (bi >= 0) {
        if (i0 == bi) { k0 = 0; i0 = -1; }
        if (i1 == bi) { k1 = 0; i1 = -1; }
      }
      if (lane == 0) {
        if (bi >= 0 && bk != 0) {
          sh.top_tok[k] = sh.ctok[bi];
          sh.top_p[k] = __longlong_as_double((long long)(bk - 1));
        } else {
          sh.top_tok[k] = -1;
          sh.top_p[k] = 0.0;
        }
      }
    }
#ifdef VP_DRAFT_TRACE
    if (tid == 0) sh.tacc[24] = clock64();
#endif
  }
  __syncthreads();
  DR_T(sh, 10);
}

// One draft tree of at most B nodes (B <= 15) with `branch` (<= 8) children per expansion, after
// the committed tokens out0[0 .. st->step), written as the next pass's tree buffer.
__global__ void __launch_bounds__(DR_THREADS, 1) k_draft(DraftTab T, DraftReq R, const int32_t* out0,
                                                        const vp_state* st, int lo0_given, int B, int branch,
                                                        DraftOut O) {
  extern __shared__ __align__(16) uint8_t dr_smem[];
  DrShared& sh = *reinterpret_cast<DrShared*>(dr_smem);
  const int tid = threadIdx.x;
  const int lo0 = st ? __ldcg(&st->step) : lo0_given;
  const bool done = st ? __ldcg(&st->done) != 0 : false;
  for (int i = tid; i < DR_WORDS; i += DR_THREADS) {
    sh.used[i] = 0u;
    sh.mark[i] = 0u;
    sh.prm[i] = 0u;
  }
  if (tid < DR_SUMW) sh.msum[tid] = 0u;
  if (tid == 0) { sh.capped = 0; sh.hn = 0; sh.hctr = 0; sh.nodes = 0; }
#ifdef VP_DRAFT_TRACE
  if (tid < 32) sh.tacc[tid] = 0ull;
  if (tid == 0) sh.tlast = globaltimer();
#endif
  // stage what every context reads: the output, the prompt, the distinct prompt ids with their
  // copy propensities, the MLP
  const bool st_out = lo0 <= DR_OUT_CAP, st_pr = R.np <= DR_PROMPT_CAP, st_cp = R.ncopy <= DR_COPY_CAP;
  if (st_out)
    for (int i = tid; i < lo0; i += DR_THREADS) sh.outs[i] = out0[i];
  if (st_pr)
    for (int i = tid; i < R.np; i += DR_THREADS) sh.prs[i] = R.P[i];
  if (st_cp)
    for (int i = tid; i < R.ncopy; i += DR_THREADS) {
      const int t = R.copy[i];
      sh.cps[i] = t;
      const int j = dr_find(T.prop, T.n_prop, (uint32_t)t, dr_rtok);
      sh.cpp[i] = j >= 0 ? T.prop[j].v : __int_as_float(0x7fc00000);  // NaN: not in the table
      const double pt = j >= 0 ? (double)T.prop[j].v : 0.2;
      sh.cplg[i] = log(pt / (1.0 - pt)) / 4.0;
    }
  const bool st_as = R.nas <= DR_AS_CAP && R.nascand <= DR_AS_CAP;
  if (st_as) {
    for (int i = tid; i < R.nas; i += DR_THREADS) {
      sh.ast[i] = R.as_tok[i];
      sh.asmx[i] = R.as_max[i];
      sh.ascn[i] = R.as_cnt[i];
    }
    for (int i = tid; i < R.nascand; i += DR_THREADS) sh.asc[i] = R.as_cand[i];
  }
  if (tid < R.nnb) sh.nbs[tid] = R.nb_score[tid];
  const int n_mlp = T.H * DR_F + 2 * T.H + 1 + DR_F;
  for (int i = tid; i < n_mlp; i += DR_THREADS) sh.mlpd[i] = (double)T.mlp[i];
  __syncthreads();
  if (st_pr) R.P = sh.prs;
  if (st_cp) {
    R.copy = sh.cps;
    R.copy_prop = sh.cpp;
    R.copy_logit = sh.cplg;
  }
  if (st_as) {
    R.as_tok = sh.ast;
    R.as_max = sh.asmx;
    R.as_cnt = sh.ascn;
    R.as_cand = sh.asc;
  }
  R.nb_score = sh.nbs;
  const int32_t* outp = st_out ? sh.outs : out0;
  int ticks = 0;  // backticks of the committed output (integer sum: any order)
  for (int i = tid; i < lo0; i += DR_THREADS) {
    const int t = outp[i];
    if (t >= 0 && t < DR_VOCAB) atomicOr(&sh.used[t >> 5], 1u << (t & 31));
    ticks += dr_flag(T, t) & 7;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ticks += __shfl_xor_sync(0xffffffffu, ticks, o);
  if ((tid & 31) == 0) sh.red_i[tid >> 5] = ticks;
  __syncthreads();
  if (tid == 0) {
    int r = 0;
    for (int w = 0; w < DR_THREADS / 32; ++w) r += sh.red_i[w];
    sh.ticks0 = r;
  }
  __syncthreads();
  DrCtx c;
  c.out0 = outp;
  c.lo0 = lo0;
  c.path = sh.path;
  // the root's candidates, then best first: pop, record, expand unless a stop token or full. One
  // call site of dr_expand (the root is the expansion of node -1 with key -1: its children's keys
  // are -p exactly), so the kernel's code holds one copy of it.
  if (!done) {
    const int ntop = O.exp_tok ? 8 : branch;  // the debug block records all 8
    int exp_i = 0;
    double key = -1.0;
    int node = -1;
    c.np = 0;
    for (;;) {
      dr_expand(T, R, c, sh, ntop);
      if (tid == 0) {
        for (int k = 0; k < branch; ++k)
          if (sh.top_tok[k] >= 0 && sh.hn < DR_HEAP) {
            const int h = sh.hn++;
            sh.hk[h] = key * sh.top_p[k]; sh.hseq[h] = sh.hctr++; sh.hpar[h] = node; sh.htok[h] = sh.top_tok[k];
          }
        if (O.exp_tok && exp_i < 16)
          for (int k = 0; k < 8; ++k) { O.exp_tok[exp_i * 8 + k] = sh.top_tok[k]; O.exp_p[exp_i * 8 + k] = sh.top_p[k]; }
      }
      ++exp_i;
      __syncthreads();
      int go = 1;
      while (go == 1) {
        if (tid < 32) {
          // warp 0 finds the smallest (key, seq) of the queue; thread 0 pops it
          const bool can = sh.hn > 0 && sh.nodes < B;
          int b = -1;
          if (can) {
            // smallest key first, then the smallest sequence number: as the largest complemented
            // order-preserving key, then the lowest sequence among the lanes that hold it
            unsigned long long bk = 0;
            int bs = 0x7fffffff, bl = -1;
            for (int h = tid; h < sh.hn; h += 32) {
              const unsigned long long u = ~dr_ord(sh.hk[h]);
              if (bl < 0 || u > bk || (u == bk && sh.hseq[h] < bs)) { bl = h; bk = u; bs = sh.hseq[h]; }
            }
            const unsigned long long m = warp_max_u64(bl >= 0 ? bk : 0ull);
            const bool at = bl >= 0 && bk == m;
            const unsigned smin = __reduce_min_sync(0xffffffffu, at ? (unsigned)bs : 0xffffffffu);
            b = __reduce_max_sync(0xffffffffu, (at && (unsigned)bs == smin) ? bl : -1);
          }
          if (tid == 0) sh.go = 0;
          if (tid == 0 && can) {
            const double kb = sh.hk[b];
            const int par = sh.hpar[b], tok = sh.htok[b];
            --sh.hn;
            sh.hk[b] = sh.hk[sh.hn]; sh.hseq[b] = sh.hseq[sh.hn]; sh.hpar[b] = sh.hpar[sh.hn]; sh.htok[b] = sh.htok[sh.hn];
            const int nd = sh.nodes++;
            sh.npar[nd] = par; sh.ntok[nd] = tok;
            sh.cur = nd;
            sh.red_d[0] = kb;
            if (tok != 151645 && tok != 151643 && sh.nodes < B) {
              // the node's path from the root
              int d = 0, v = nd;
              int rev[16];
              while (v >= 0) { rev[d++] = sh.ntok[v]; v = sh.npar[v]; }
              for (int i = 0; i < d; ++i) sh.path[i] = rev[d - 1 - i];
              sh.npath = d;
              sh.go = 2;
            } else {
              sh.go = 1;
            }
          }
        }
        __syncthreads();
        go = sh.go;
        if (go == 2) {
          key = sh.red_d[0];
          node = sh.cur;
          c.np = sh.npath;
        }
        __syncthreads();
      }
      if (go == 0) break;
    }
  }
  // the tree buffer: row 0 the last committed token, row i + 1 node i
  if (tid == 0) {
    const int n = done ? 1 : 1 + sh.nodes;
    int depth[16], anc[16];
    depth[0] = 0; anc[0] = 1;
    O.tree[VP_TR_N] = n;
    for (int r = 0; r < ROWS; ++r) {
      int d = 0, p = r - 1, tk = 0, a = 0;
      if (r == 0) { p = -1; tk = lo0 >= 1 ? out0[lo0 - 1] : 0; a = 1; }
      else if (r < n) {
        p = sh.npar[r - 1] + 1; tk = sh.ntok[r - 1]; d = depth[p] + 1; a = anc[p] | (1 << r);
      } else { p = 0; d = 0; a = 0; }
      if (r < 16) { depth[r] = d; anc[r] = a; }
      O.tree[VP_TR_DEPTH + r] = d;
      O.tree[VP_TR_PARENT + r] = r == 0 ? -1 : p;
      O.tree[VP_TR_TOK + r] = tk;
      O.tree[VP_TR_ANC + r] = a;
    }
    if (O.parents)
      for (int i = 0; i < 15; ++i) {
        O.parents[i] = i < (done ? 0 : sh.nodes) ? sh.npar[i] : -2;
        O.tokens[i] = i < (done ? 0 : sh.nodes) ? sh.ntok[i] : -1;
      }
    if (O.status) *O.status = sh.capped;
  }
#ifdef VP_DRAFT_TRACE
  DR_T(sh, 12);
  if (tid < 32) g_dr_trace[tid] = sh.tacc[tid];
#endif
}

}  // namespace vp
