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

struct DrShared {
  uint32_t used[DR_WORDS];                 // bitset of the committed output's tokens
  unsigned long long cand[DR_MAX_CAND];    // (token << 32) | source bits, sorted and merged
  double prob[DR_MAX_CAND];
  unsigned long long hsh[DR_MAXM_MAX + 1]; // key of the context's last n tokens
  int dist_tot[DR_N_MAX + 1], dist_first[DR_N_MAX + 1], dist_n[DR_N_MAX + 1];
  int long_n, supp3, supp10, top_long, ent_low;
  int vote_tok[DR_MAX_NB], vote_n[DR_MAX_NB];
  int path[16], npath;
  int ncand, red_i[DR_THREADS / 32];
  double red_d[DR_THREADS / 32];
  int self_n, self_tok, pr_n, pr_first_e, first_unused, ticks0, capped;
  double c1, c2;
  // best-first queue and the tree
  double hk[DR_HEAP]; int hseq[DR_HEAP], hpar[DR_HEAP], htok[DR_HEAP], hn, hctr;
  int npar[16], ntok[16], nodes, cur, go;
  int top_tok[8]; double top_p[8];
};

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

// Block reductions (256 threads) with a fixed combination order.
__device__ __forceinline__ int dr_max_i(int v, DrShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sh.red_i[threadIdx.x >> 5] = v;
  __syncthreads();
  int r = sh.red_i[0];
  for (int w = 1; w < DR_THREADS / 32; ++w) r = max(r, sh.red_i[w]);
  __syncthreads();
  return r;
}
__device__ __forceinline__ int dr_min_i(int v, DrShared& sh) { return -dr_max_i(-v, sh); }
__device__ __forceinline__ double dr_max_d(double v, DrShared& sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmax(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) sh.red_d[threadIdx.x >> 5] = v;
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

// Longest common suffix of seq[0..e) and the output (both end-aligned), at most cap.
template <typename Seq>
__device__ __forceinline__ int dr_suffix(const Seq& s, int e, const DrCtx& c, int cap) {
  const int lo = c.lo();
  int k = 0;
  while (k < cap && k < e && s(e - 1 - k) == c.out(lo - 1 - k)) ++k;
  return k;
}

// Candidates and probabilities of the next token after the context; leaves the top 8 (probability
// descending, token ascending) in sh.top_tok / top_p (-1: fewer candidates).
__device__ void dr_expand(const DraftTab& T, const DraftReq& R, const DrCtx& c, DrShared& sh) {
  const int tid = threadIdx.x;
  const int L = c.L(), lo = c.lo();
  const int nmax = max(T.N, T.MAXM);
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
  if (tid == 0) { sh.ncand = 0; sh.self_n = 0; sh.pr_n = 0; }
  __syncthreads();
  // n-gram distributions of orders 1..min(N, L)
  if (tid >= 1 && tid <= T.N) {
    int tot = -1, first = 0, n = 0;
    if (tid <= L) {
      const int i = dr_find(T.ngky, T.n_ng, sh.hsh[tid], dr_u64);
      if (i >= 0) { tot = (int)T.ngvl[i].a; first = (int)(T.ngvl[i].b >> 3); n = (int)(T.ngvl[i].b & 7u); }
    }
    sh.dist_tot[tid] = tot; sh.dist_first[tid] = first; sh.dist_n[tid] = n;
  }
  // neighbours: the longest context suffix in each document's index gives its vote
  if (tid < R.nnb) {
    int tok = -1, got = 0;
    const int k0 = R.nb_key_off[tid], k1 = R.nb_key_off[tid + 1];
    for (int n = min(T.MAXM, L); n >= 1 && tok < 0; --n) {
      const int i = dr_find(R.nb_keys + k0, k1 - k0, sh.hsh[n], dr_u64);
      if (i >= 0) { tok = R.nb_seq[R.nb_seq_off[tid] + R.nb_pos[k0 + i]]; got = n; }
    }
    sh.vote_tok[tid] = tok; sh.vote_n[tid] = got;
  }
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
  // prompt lookup: every occurrence of the longest suffix of the output found in the prompt
  best = 0;
  const int capp = min(T.MAXM, lo);
  for (int e = 1 + tid; e <= R.np - 1; e += DR_THREADS)
    best = max(best, dr_suffix([&](int i) { return R.P[i]; }, e, c, capp));
  const int pr_n = dr_max_i(best, sh);
  if (tid == 0) sh.pr_n = pr_n;
  __syncthreads();
  // the candidate list: (token << 32) | source bits, merged after sorting
  auto push = [&](int tok, uint32_t bits) {
    const int k = atomicAdd(&sh.ncand, 1);
    if (k < DR_MAX_CAND) sh.cand[k] = ((unsigned long long)(uint32_t)tok << 32) | bits;
  };
  if (pr_n > 0) {
    int first = 0x7fffffff;
    for (int e = 1 + tid; e <= R.np - 1; e += DR_THREADS)
      if (dr_suffix([&](int i) { return R.P[i]; }, e, c, capp) >= pr_n) { push(R.P[e], DS_PR); first = min(first, e); }
    first = dr_min_i(first, sh);
    if (tid == 0) { sh.pr_first_e = first; push(R.P[first], DS_PRFIRST); }
  }
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
      const DrPair* top = T.ngnx + sh.dist_first[ln];
      sh.top_long = (int)top[0].a;
      double ent = 0.0;
      const double tot = (double)sh.dist_tot[ln];
      for (int i = 0; i < sh.dist_n[ln]; ++i) {
        const double q = (double)top[i].b / tot;
        ent = ent + q * log(q);
      }
      sh.ent_low = -ent < 0.3;
    }
    for (int n = 1; n <= T.N; ++n)
      if (sh.dist_tot[n] >= 0)
        for (int i = 0; i < sh.dist_n[n]; ++i) push((int)T.ngnx[sh.dist_first[n] + i].a, DS_NG);
    if (sh.self_n > 0) push(sh.self_tok, DS_SELF);
    for (int r = 0; r < R.nnb; ++r)
      if (sh.vote_tok[r] >= 0) push(sh.vote_tok[r], DS_NB);
    const int t1 = c.ctx(L - 1), t2 = c.ctx(L - 2);
    const int i1 = dr_find(T.cc1, T.n_cc1, (uint32_t)t1, dr_rtok);
    sh.c1 = i1 >= 0 ? (double)T.cc1[i1].v : 0.1;
    const int i2 = dr_find(T.cc2, T.n_cc2, ((unsigned long long)(uint32_t)t2 << 32) | (uint32_t)t1, dr_r2key);
    sh.c2 = i2 >= 0 ? (double)T.cc2[i2].v : 0.1;
  }
  // the first prompt id not in the output whose copy propensity exceeds 0.3
  {
    int fu = 0x7fffffff;
    for (int j = tid; j < R.np; j += DR_THREADS)
      if (!dr_used(sh, c, R.P[j]) && dr_prop(T, R.P[j], 0.2) > 0.3) fu = min(fu, j);
    fu = dr_min_i(fu, sh);
    if (tid == 0) sh.first_unused = fu < R.np ? R.P[fu] : -1;
  }
  for (int j = tid; j < R.ncopy; j += DR_THREADS) push(R.copy[j], DS_COPY);
  for (int j = tid; j < R.nascand; j += DR_THREADS) push(R.as_cand[j], DS_ASC);
  __syncthreads();
  // sort (bitonic, padded with the largest key) and merge equal tokens
  const int n_raw = sh.ncand;
  if (tid == 0 && n_raw > DR_MAX_CAND) sh.capped = 1;
  const int nr = min(n_raw, DR_MAX_CAND);
  int np2 = 1;
  while (np2 < nr) np2 <<= 1;
  for (int i = nr + tid; i < np2; i += DR_THREADS) sh.cand[i] = ~0ull;
  __syncthreads();
  for (int k = 2; k <= np2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < np2; i += DR_THREADS) {
        const int ixj = i ^ j;
        if (ixj > i) {
          const unsigned long long a = sh.cand[i], b = sh.cand[ixj];
          if (((i & k) == 0) == (a > b)) { sh.cand[i] = b; sh.cand[ixj] = a; }
        }
      }
      __syncthreads();
    }
  if (tid == 0) {
    int m = 0;
    for (int i = 0; i < nr; ++i) {
      const unsigned long long v = sh.cand[i];
      if (m > 0 && (sh.cand[m - 1] >> 32) == (v >> 32)) sh.cand[m - 1] |= v & 0xffffffffull;
      else sh.cand[m++] = v;
    }
    sh.ncand = m;
  }
  __syncthreads();
  const int nc = sh.ncand;
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
  const float* W1 = T.mlp;
  const float* b1 = W1 + T.H * DR_F;
  const float* W2 = b1 + T.H;
  const double b2 = (double)W2[T.H];
  const float* WL = W2 + T.H + 1;
  for (int ci = tid; ci < nc; ci += DR_THREADS) {
    const int tok = (int)(sh.cand[ci] >> 32);
    const uint32_t src = (uint32_t)sh.cand[ci];
    double x[DR_F];
#pragma unroll
    for (int f = 0; f < DR_F; ++f) x[f] = 0.0;
    x[F_BIAS] = 1.0;
    for (int n = 1; n <= T.N; ++n) {
      if (sh.dist_tot[n] < 0) continue;
      const DrPair* top = T.ngnx + sh.dist_first[n];
      int cnt = 0, rank = -1;
      for (int i = 0; i < sh.dist_n[n]; ++i)
        if ((int)top[i].a == tok) { cnt = (int)top[i].b; rank = i; break; }
      if (n == sh.long_n && rank >= 1) x[rank == 1 ? F_NG_RANK2 : F_NG_RANK3PLUS] = 1.0;
      if (cnt) {
        const double p = (double)cnt / (double)sh.dist_tot[n];
        if (n <= 6) x[F_NG_P1 + n - 1] = p;
        if (n == sh.long_n) {
          x[F_NG_P_LONG] = p;
          x[F_NG_ORD_LONG] = (double)n / 6.0 * p;
          x[F_NG_LCNT_LONG] = log1p((double)cnt);
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
      int cnt = 0, mm = 0;
      for (int r = 0; r < R.nnb; ++r)
        if (sh.vote_tok[r] == tok) {
          const int m8 = min(sh.vote_n[r], 8);
          s1 = s1 + R.nb_score[r];
          s2 = s2 + R.nb_score[r] * (double)m8 / 8.0;
          ++cnt;
          mm = max(mm, m8);
          if (r == 0) { x[F_NB_TOP1] = 1.0; x[F_NB_TOP1_M] = (double)m8 / 8.0; }
        }
      x[F_NB_SUM] = s1;
      x[F_NB_MSUM] = s2;
      x[F_NB_CNT] = (double)cnt / (double)max(1, R.nnb);
      x[F_NB_MAXM] = (double)mm / 8.0;
    }
    const bool in_p = dr_find(R.copy, R.ncopy, tok, dr_i32) >= 0;
    const bool used = dr_used(sh, c, tok);
    if (src & DS_COPY) {
      const double pt = in_p ? dr_prop(T, tok, 0.2) : 0.3;
      x[F_CP_PROP] = log(pt / (1.0 - pt)) / 4.0;
      x[F_CP_CTX1] = sh.c1;
      x[F_CP_CTX2] = sh.c2;
      x[F_CP_UNUSED] = used ? 0.0 : 1.0;
      x[F_CP_FIRST_UNUSED] = tok == sh.first_unused ? 1.0 : 0.0;
      x[F_CP_SPACEVAR] = in_p ? 0.0 : 1.0;
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
    // score = W2 . relu(W1 x + b1) + b2 + WL . x
    double s = 0.0;
    for (int h = 0; h < T.H; ++h) {
      double a = 0.0;
      for (int f = 0; f < DR_F; ++f) a = fma((double)W1[h * DR_F + f], x[f], a);
      a += (double)b1[h];
      s = fma((double)W2[h], fmax(a, 0.0), s);
    }
    double lin = 0.0;
    for (int f = 0; f < DR_F; ++f) lin = fma((double)WL[f], x[f], lin);
    sh.prob[ci] = s + b2 + lin;
  }
  __syncthreads();
  // softmax with a null option of score 0
  double m = -INFINITY;
  for (int ci = tid; ci < nc; ci += DR_THREADS) m = fmax(m, sh.prob[ci]);
  m = fmax(dr_max_d(m, sh), 0.0);
  double z = 0.0;
  for (int ci = tid; ci < nc; ci += DR_THREADS) z += exp(sh.prob[ci] - m);
  z = dr_sum_d(z, sh) + exp(-m);
  for (int ci = tid; ci < nc; ci += DR_THREADS) sh.prob[ci] = exp(sh.prob[ci] - m) / z;
  __syncthreads();
  // the 8 most probable, probability descending then token ascending
  for (int k = 0; k < 8; ++k) {
    double bp = -1.0;
    int bi = -1;
    for (int ci = tid; ci < nc; ci += DR_THREADS)
      if (sh.prob[ci] > bp) { bp = sh.prob[ci]; bi = ci; }  // ascending ci = ascending token
    // reduce (p desc, index asc) across the block through packed keys on the warp, then thread 0
    for (int o = 16; o > 0; o >>= 1) {
      const double op = __shfl_xor_sync(0xffffffffu, bp, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (op > bp || (op == bp && oi >= 0 && (bi < 0 || oi < bi))) { bp = op; bi = oi; }
    }
    if ((tid & 31) == 0) { sh.red_d[tid >> 5] = bp; sh.red_i[tid >> 5] = bi; }
    __syncthreads();
    if (tid == 0) {
      double p = sh.red_d[0];
      int i = sh.red_i[0];
      for (int w = 1; w < DR_THREADS / 32; ++w)
        if (sh.red_d[w] > p || (sh.red_d[w] == p && sh.red_i[w] >= 0 && (i < 0 || sh.red_i[w] < i))) {
          p = sh.red_d[w]; i = sh.red_i[w];
        }
      if (i >= 0 && p >= 0.0) {
        sh.top_tok[k] = (int)(sh.cand[i] >> 32);
        sh.top_p[k] = p;
        sh.prob[i] = -2.0;  // taken
      } else {
        sh.top_tok[k] = -1;
        sh.top_p[k] = 0.0;
      }
    }
    __syncthreads();
  }
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
  for (int i = tid; i < DR_WORDS; i += DR_THREADS) sh.used[i] = 0u;
  if (tid == 0) { sh.capped = 0; sh.hn = 0; sh.hctr = 0; sh.nodes = 0; }
  __syncthreads();
  int ticks = 0;  // backticks of the committed output (integer sum: any order)
  for (int i = tid; i < lo0; i += DR_THREADS) {
    const int t = out0[i];
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
  c.out0 = out0;
  c.lo0 = lo0;
  c.path = sh.path;
  // the root's candidates, then best first: pop, record, expand unless a stop token or full
  int exp_i = 0;
  if (!done) {
    c.np = 0;
    dr_expand(T, R, c, sh);
    if (tid == 0) {
      for (int k = 0; k < branch; ++k)
        if (sh.top_tok[k] >= 0) {
          const int h = sh.hn++;
          sh.hk[h] = -sh.top_p[k]; sh.hseq[h] = sh.hctr++; sh.hpar[h] = -1; sh.htok[h] = sh.top_tok[k];
        }
      if (O.exp_tok)
        for (int k = 0; k < 8; ++k) { O.exp_tok[k] = sh.top_tok[k]; O.exp_p[k] = sh.top_p[k]; }
    }
    ++exp_i;
    __syncthreads();
    for (;;) {
      if (tid == 0) {
        sh.go = 0;
        if (sh.hn > 0 && sh.nodes < B) {
          // pop the smallest (key, seq)
          int b = 0;
          for (int h = 1; h < sh.hn; ++h)
            if (sh.hk[h] < sh.hk[b] || (sh.hk[h] == sh.hk[b] && sh.hseq[h] < sh.hseq[b])) b = h;
          const double key = sh.hk[b];
          const int par = sh.hpar[b], tok = sh.htok[b];
          --sh.hn;
          sh.hk[b] = sh.hk[sh.hn]; sh.hseq[b] = sh.hseq[sh.hn]; sh.hpar[b] = sh.hpar[sh.hn]; sh.htok[b] = sh.htok[sh.hn];
          const int node = sh.nodes++;
          sh.npar[node] = par; sh.ntok[node] = tok;
          sh.cur = node;
          sh.red_d[0] = key;
          if (tok != 151645 && tok != 151643 && sh.nodes < B) {
            // the node's path from the root
            int d = 0, v = node;
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
      const int go = sh.go;
      if (go == 0) break;
      if (go == 2) {
        const double key = sh.red_d[0];
        const int node = sh.cur;
        __syncthreads();
        c.np = sh.npath;
        dr_expand(T, R, c, sh);
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
      }
      __syncthreads();
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
}

}  // namespace vp
