// Accept / commit, request set-up and weight packing kernels.
#pragma once
#include "vp_common.cuh"

namespace vp {

constexpr int COMMIT_THREADS = CONS_THREADS;

struct CommitParams {
  const float* pval;  // [16][nparts] argmax partials (value)
  const int* pidx;    // [16][nparts] (id, lowest on ties)
  int nparts;
  Scratch s;
};

// Greedy accept + commit (k_commit_spec, Shaders.swift:254-365, and k_commit :194-244), run by the
// 512 compute threads of one CTA:
//  1. g[t] = argmax of pass row vrow0+t over the argmax partials, lowest id on ties (:281-306).
//  2. Tree: from the root, repeatedly take the first row whose parent is the current row and whose
//     draft equals the current row's argmax (:311-320). The root's argmax is always committed.
//  3. Commit g along the path to out_tokens, stopping at EOS or max_steps (:326-333).
//  4. pos += m + 1 (verify) or += prompt length (prefill, :335-338).
//  5. KV compaction: accepted row path[k-1] moves from slot pos0+path[k-1] to pos0+k in every
//     layer; it was already rotated for position pos0+k (its depth is k) (:351-365). The moves
//     go in batches of four k: a batch reads all its sources before writing its destinations, and
//     its destinations (pos0+k, k <= the batch's last) lie below every later batch's sources
//     (pos0+path[k'-1] >= pos0+k', since path rows strictly increase), so no read sees a moved row.
//     Each thread keeps the same 16-byte words in every batch, so batches need no barrier.
__device__ void commit_body(const Scratch& s, const float* pval, const int* pidx, int nparts) {
  vp_state* st = s.st;
  const RowInfo* ri = s.ri;
  if (!ri->live || __ldcg(&st->done)) return;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nthr = CONS_THREADS;
  const int nwarps = nthr >> 5;
  __shared__ int g[ROWS];
  __shared__ int path[ROWS];
  __shared__ int sTree[VP_TREE_INTS];
  __shared__ int sNpath, sPos0;
  const int nv = st->nver, r0 = st->vrow0;
  // the tree buffer comes in with the partials, so the walk below reads shared memory only
  if (tid < VP_TREE_INTS) sTree[tid] = __ldcg(s.tree + tid);
  // one warp per row: argmax over the partials, lowest id on ties
  for (int t = warp; t < nv; t += nwarps) {
    const float* pv = pval + (size_t)(r0 + t) * nparts;
    const int* pi = pidx + (size_t)(r0 + t) * nparts;
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = lane; i < nparts; i += 32) {
      const float v = __ldcg(pv + i);
      const int id = __ldcg(pi + i);
      if (v > best || (v == best && id < bi)) { best = v; bi = id; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > best || (ov == best && oi < bi)) { best = ov; bi = oi; }
    }
    if (lane == 0) g[t] = bi;
  }
  cons_sync();
  if (tid == 0) {
    int m = 0;
    const bool tree = ri->mode == 0 && nv > 1;
    if (tree) {
      int cur = 0;
      for (;;) {
        int c = -1;
        for (int i = 1; i < nv; ++i)
          if (sTree[VP_TR_PARENT + i] == cur && sTree[VP_TR_TOK + i] == g[cur]) { c = i; break; }
        if (c < 0) break;
        path[m++] = c;
        cur = c;
      }
    }
    // the state is read once and written back once: the serial part runs on registers (through
    // the pointer every field access would be a dependent round trip, since the token stores
    // below may alias it)
    const int pos = __ldcg(&st->pos), step0 = __ldcg(&st->step), eos0 = __ldcg(&st->eos0);
    const int eos1 = __ldcg(&st->eos1), maxsteps = __ldcg(&st->maxsteps), advance = __ldcg(&st->advance);
    const int passes = __ldcg(&st->passes), accepted = __ldcg(&st->accepted);
    bool stop = false, overflow = false;
    int last = __ldcg(&st->last_token), nc = 0, step = step0;
    for (int i = 0; i <= m && !stop; ++i) {
      const int tok = g[i == 0 ? 0 : path[i - 1]];
      if (step >= s.max_steps) { overflow = true; stop = true; break; }
      s.out_tokens[step] = tok;
      if (s.pass_tok) s.pass_tok[nc] = tok;
      ++nc;
      ++step;
      last = tok;
      if (tok == eos0 || tok == eos1 || step >= maxsteps) stop = true;
    }
    if (s.pass_tok)
      for (int i = nc; i < ROWS; ++i) s.pass_tok[i] = -1;
    sPos0 = pos;
    sNpath = tree ? m : 0;
    st->passes = passes + 1;
    st->accepted = accepted + m;
    st->step = step;
    st->pos = pos + (ri->mode == 1 ? advance : m + 1);
    st->last_token = last;
    if (overflow) atomicOr(&st->err, VP_DEV_ERR_STEPS);
    if (stop) st->done = 1;
  }
  cons_sync();
  const int np = sNpath, pos0 = sPos0;
  // 2 caches x layers x 2 KV heads x 64 halves, moved as 16-byte words (8 per row)
  const int words = 2 * s.n_layers * NKV * (HD / 8);
  for (int k0 = 1; k0 <= np; k0 += 4) {
    const int kn = min(4, np - k0 + 1);
    for (int w = tid; w < words; w += nthr) {
      const int cache = w / (s.n_layers * NKV * 8);
      const int rem = w % (s.n_layers * NKV * 8);
      const int lh = rem / 8, part = rem % 8;
      __half* base = (cache ? s.vc : s.kc) + (size_t)lh * s.max_ctx * HD + part * 8;
      uint4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < kn) v[j] = __ldcg(reinterpret_cast<const uint4*>(base + (size_t)(pos0 + path[k0 + j - 1]) * HD));
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (j < kn && path[k0 + j - 1] != k0 + j)
          *reinterpret_cast<uint4*>(base + (size_t)(pos0 + k0 + j) * HD) = v[j];
    }
  }
}

__global__ void __launch_bounds__(COMMIT_THREADS) k_commit(CommitParams p) {
  commit_body(p.s, p.pval, p.pidx, p.nparts);
}

// Request set-up (Engine.generate, Engine.swift:945-964): one thread.
__global__ void k_begin(vp_state* st, int32_t* out_tokens, int max_steps_cap, int cached,
                        int max_new, int eos0, int eos1, int maxctx, int last_token) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  for (int j = i; j < max_steps_cap; j += gridDim.x * blockDim.x) out_tokens[j] = -1;
  if (i == 0) {
    vp_state z = {};
    z.pos = cached;
    z.n = 0;
    z.maxctx = maxctx;
    z.maxsteps = max_new;
    z.eos0 = eos0;
    z.eos1 = eos1;
    z.nver = 1;
    z.last_token = last_token;
    *st = z;
  }
}

// Chain tree from a draft list: rows 0..nd, parent i-1, depth i (Shaders.swift:322 semantics).
__global__ void k_chain_tree(int32_t* tree, const int32_t* drafts, int nd) {
  const int i = threadIdx.x;
  if (i == 0) tree[VP_TR_N] = nd + 1;
  if (i < ROWS) {
    tree[VP_TR_DEPTH + i] = i;
    tree[VP_TR_PARENT + i] = i - 1;
    tree[VP_TR_TOK + i] = (i >= 1 && i <= nd) ? drafts[i - 1] : 0;
    tree[VP_TR_ANC + i] = (int)((2u << i) - 1u);
  }
}

// ---------------------------------------------------------------------------------------------
// Weight packing: standard layouts -> fragment-ordered tiles (see vp_common.cuh).

__device__ __forceinline__ int src_row(int kind, int rb, int r) {
  if (kind == VP_MAT_QKV) {
    const int head = rb >> 2, jj = rb & 3;
    return head * HD + (r < 8 ? 8 * jj + r : 32 + 8 * jj + (r - 8));
  }
  if (kind == VP_MAT_GATEUP) return r < 8 ? rb * 8 + r : F + rb * 8 + (r - 8);
  return rb * 16 + r;
}

// One thread per (tile, lane); lane 32 of each tile writes the scale block.
template <int FMT>
__global__ void k_pack(int kind, int rows, int cols, const uint8_t* codes, const uint8_t* scales,
                       uint8_t* out) {
  constexpr int TB = tile_bytes(FMT);
  const int ng = cols / GS;
  const long long ntiles = (long long)(rows / 16) * ng;
  const long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= ntiles * 33) return;
  const long long tileI = idx / 33;
  const int lane = (int)(idx % 33);
  const int rb = (int)(tileI / ng), G = (int)(tileI % ng);
  uint8_t* tile = out + tileI * TB;
  if (lane == 32) {
    for (int r = 0; r < 16; ++r) {
      const int g = r & 7, upper = r >> 3;
      const int sr = src_row(kind, rb, r);
      if (FMT == VP_FMT_Q4) {
        const uint32_t v = reinterpret_cast<const uint32_t*>(scales)[(size_t)sr * ng + G];
        reinterpret_cast<uint32_t*>(tile + 512)[g * 2 + upper] = v;
      } else if (FMT == VP_FMT_Q8) {
        const uint16_t v = reinterpret_cast<const uint16_t*>(scales)[(size_t)sr * ng + G];
        reinterpret_cast<uint16_t*>(tile + 1024)[g * 2 + upper] = v;
      } else if (FMT == VP_FMT_Q8G32) {  // scales [rows][cols/32]: both halves of the tile
        for (int h = 0; h < 2; ++h) {
          const uint16_t v = reinterpret_cast<const uint16_t*>(scales)[(size_t)sr * (2 * ng) + 2 * G + h];
          reinterpret_cast<uint16_t*>(tile + 1024)[g * 4 + h * 2 + upper] = v;
        }
      }
    }
    return;
  }
  const int g = lane >> 2, t4 = lane & 3;
  for (int j = 0; j < 4; ++j) {
    // a = reg*2 + upper: element (row g + 8*upper, col 16j + 8*reg + 2*t4 + hi)
    if (FMT == VP_FMT_Q4) {
      uint32_t w = 0;
      for (int a = 0; a < 4; ++a)
        for (int hi = 0; hi < 2; ++hi) {
          const int sr = src_row(kind, rb, g + 8 * (a & 1));
          const int k = G * GS + 16 * j + 8 * (a >> 1) + 2 * t4 + hi;
          const uint8_t b = codes[(size_t)sr * (cols / 2) + (k >> 1)];
          const uint32_t q = (k & 1) ? (b >> 4) : (b & 15);
          w |= q << ((hi ? 16 : 0) + 4 * a);
        }
      reinterpret_cast<uint32_t*>(tile + lane * 16)[j] = w;
    } else if (fmt_is_q8(FMT)) {
      uint8_t bytes[8];
      for (int a = 0; a < 4; ++a)
        for (int hi = 0; hi < 2; ++hi) {
          const int sr = src_row(kind, rb, g + 8 * (a & 1));
          const int k = G * GS + 16 * j + 8 * (a >> 1) + 2 * t4 + hi;
          bytes[(a >> 1) * 4 + (a & 1) * 2 + hi] = codes[(size_t)sr * cols + k];
        }
      for (int b = 0; b < 8; ++b) tile[lane * 32 + j * 8 + b] = bytes[b];
    } else {
      for (int a = 0; a < 4; ++a)
        for (int hi = 0; hi < 2; ++hi) {
          const int sr = src_row(kind, rb, g + 8 * (a & 1));
          const int k = G * GS + 16 * j + 8 * (a >> 1) + 2 * t4 + hi;
          reinterpret_cast<uint16_t*>(tile + lane * 64 + j * 16 + a * 4)[hi] =
              reinterpret_cast<const uint16_t*>(codes)[(size_t)sr * cols + k];
        }
    }
  }
}

}  // namespace vp
