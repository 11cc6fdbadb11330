// C ABI of the device drafter (include/vpass.h, vp_drafter_*): the ILDRAFT1 table parsed on the host
// and copied to device memory, the request context the host builds at request start, and the
// k_draft launch (vp_draft.cuh).
//
// Replaces the reference's ILDraft.swift (table load :39-60, request context :138) and the encode
// of k_ildraft (Engine.swift, between verify passes).
#include <cuda_runtime.h>

#include <cstring>
#include <string>
#include <vector>

#include "vp_draft.cuh"

using namespace vp;

// The library's error text (vp_last_error), kept by vpass.cu.
void vp_set_last_error(const std::string& msg);

namespace {

int dfail(int code, const std::string& msg) {
  vp_set_last_error(msg);
  return code;
}

#define VD_CUDA(call)                                                                   \
  do {                                                                                  \
    cudaError_t e_ = (call);                                                            \
    if (e_ != cudaSuccess) return dfail(VP_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_)); \
  } while (0)

struct Section {
  uint32_t count = 0;
  uint64_t off = 0;
  bool present = false;
};

}  // namespace

struct vp_drafter {
  int device = 0;
  DraftTab tab{};
  std::vector<void*> table_allocs;
  void* req_buf = nullptr;
  size_t req_cap = 0;
  DraftReq req{};
  bool have_req = false;
  int knb = 0;
  uint64_t gen = 0;  // requests begun so far: a step graph captured one request's pointers
};

// A replayable CUDA graph of a pass or of a decode step (see vpass.h).
struct vp_graph {
  cudaGraphExec_t exec = nullptr;
  const vp_drafter* d = nullptr;  // step graphs: the drafter and the request they captured
  uint64_t gen = 0;
  int device = 0;
};

extern "C" {

void vp_drafter_destroy(vp_drafter* d) {
  if (!d) return;
  cudaSetDevice(d->device);
  for (void* p : d->table_allocs) cudaFree(p);
  if (d->req_buf) cudaFree(d->req_buf);
  delete d;
}

int vp_drafter_create(const void* table, size_t bytes, int32_t device, vp_drafter** out) {
  if (!table || !out) return dfail(VP_ERR_ARG, "null argument");
  *out = nullptr;
  const uint8_t* b = static_cast<const uint8_t*>(table);
  if (bytes < 64 || std::memcmp(b, "ILDRAFT1", 8) != 0) return dfail(VP_ERR_ARG, "not an ILDRAFT1 table");
  uint32_t h[14];
  std::memcpy(h, b + 8, sizeof(h));
  const uint32_t version = h[0], nsec = h[1], N = h[2], MAXM = h[5], F = h[6], H = h[7], flags = h[10];
  if (version != 1) return dfail(VP_ERR_ARG, "ILDRAFT1 version is not 1");
  if (F != DR_F) return dfail(VP_ERR_ARG, "the table's feature count is not 53");
  if (H < 1 || H > DR_H_MAX || N < 1 || N > DR_N_MAX || MAXM < 1 || MAXM > DR_MAXM_MAX)
    return dfail(VP_ERR_ARG, "table sizes outside what the kernel supports (H <= 32, N <= 8, MAXM <= 16)");
  if (64 + 16ull * nsec > bytes) return dfail(VP_ERR_ARG, "section directory outside the table");
  auto sec = [&](const char* tag) {
    Section s;
    for (uint32_t i = 0; i < nsec; ++i) {
      const uint8_t* e = b + 64 + 16 * i;
      if (std::memcmp(e, tag, 4) == 0) {
        std::memcpy(&s.count, e + 4, 4);
        std::memcpy(&s.off, e + 8, 8);
        s.present = true;
      }
    }
    return s;
  };
  const Section ngky = sec("NGKY"), ngvl = sec("NGVL"), ngnx = sec("NGNX"), cptk = sec("CPTK"), cpc1 = sec("CPC1"),
                cpc2 = sec("CPC2"), tfls = sec("TFLS"), tflg = sec("TFLG"), mlp = sec("MLP0");
  auto fits = [&](const Section& s, size_t rec) { return !s.present || s.off + (uint64_t)s.count * rec <= bytes; };
  if (!ngky.present || !ngvl.present || !ngnx.present || !mlp.present || ngky.count != ngvl.count)
    return dfail(VP_ERR_ARG, "n-gram or MLP sections missing");
  if (!fits(ngky, 8) || !fits(ngvl, 8) || !fits(ngnx, 8) || !fits(cptk, 8) || !fits(cpc1, 8) || !fits(cpc2, 16) ||
      !fits(tfls, 8) || !fits(tflg, 1) || !fits(mlp, 4))
    return dfail(VP_ERR_ARG, "a section runs past the end of the table");
  if (mlp.count < H * DR_F + 2 * H + 1 + DR_F) return dfail(VP_ERR_ARG, "MLP section too short");

  vp_drafter* d = new vp_drafter();
  d->device = device;
  cudaError_t e = cudaSetDevice(device);
  // k_draft keeps the staged request and the candidate bitsets in ~150 KB of shared memory
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(k_draft, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(DrShared));
  if (e != cudaSuccess) { delete d; return dfail(VP_ERR_CUDA, cudaGetErrorString(e)); }
  auto upload = [&](const void* src, size_t n, void** dst) -> int {
    void* p = nullptr;
    cudaError_t err = cudaMalloc(&p, n ? n : 16);
    if (err != cudaSuccess) return dfail(VP_ERR_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(err));
    d->table_allocs.push_back(p);
    if (n) {
      err = cudaMemcpy(p, src, n, cudaMemcpyHostToDevice);
      if (err != cudaSuccess) return dfail(VP_ERR_CUDA, std::string("cudaMemcpy: ") + cudaGetErrorString(err));
    }
    *dst = p;
    return VP_OK;
  };
  DraftTab& T = d->tab;
  void* p = nullptr;
  int r = VP_OK;
#define UP(S, REC, FIELD, CNT)                                                            \
  if (!r) {                                                                              \
    r = upload(b + (S).off, (S).present ? (size_t)(S).count * (REC) : 0, &p);            \
    T.FIELD = reinterpret_cast<decltype(T.FIELD)>(p);                                    \
    CNT;                                                                                 \
  }
  UP(ngky, 8, ngky, T.n_ng = (int)ngky.count);
  UP(ngvl, 8, ngvl, (void)0);
  UP(ngnx, 8, ngnx, (void)0);
  UP(cptk, 8, prop, T.n_prop = cptk.present ? (int)cptk.count : 0);
  UP(cpc1, 8, cc1, T.n_cc1 = cpc1.present ? (int)cpc1.count : 0);
  UP(cpc2, 16, cc2, T.n_cc2 = cpc2.present ? (int)cpc2.count : 0);
  UP(mlp, 4, mlp, (void)0);
#undef UP
  if (!r) {
    // dense token flags: TFLS holds (token, flags) for the tokens with flags; TFLG a dense prefix
    std::vector<uint8_t> fl(DR_VOCAB, 0);
    if (tfls.present)
      for (uint32_t i = 0; i < tfls.count; ++i) {
        uint32_t tk, v;
        std::memcpy(&tk, b + tfls.off + 8ull * i, 4);
        std::memcpy(&v, b + tfls.off + 8ull * i + 4, 4);
        if (tk < (uint32_t)DR_VOCAB) fl[tk] = (uint8_t)v;
      }
    else if (tflg.present)
      std::memcpy(fl.data(), b + tflg.off, std::min<size_t>(tflg.count, DR_VOCAB));
    r = upload(fl.data(), fl.size(), &p);
    T.tflg = static_cast<const uint8_t*>(p);
  }
  if (r) { vp_drafter_destroy(d); return r; }
  T.N = (int)N;
  T.MAXM = (int)MAXM;
  T.H = (int)H;
  T.flags = (int)flags;
  *out = d;
  return VP_OK;
}

int vp_drafter_begin(vp_drafter* d, const vp_draft_request* q) {
  if (!d || !q) return dfail(VP_ERR_ARG, "null argument");
  if (q->n_prompt < 0 || q->n_prompt > VP_DRAFT_MAX_PROMPT || q->n_copy < 0 || q->n_copy > q->n_prompt)
    return dfail(VP_ERR_ARG, "prompt longer than VP_DRAFT_MAX_PROMPT or bad copy count");
  if (q->n_nb < 0 || q->n_nb > DR_MAX_NB) return dfail(VP_ERR_ARG, "at most 16 neighbour documents");
  if (q->n_as < 0 || q->n_as_cand < 0) return dfail(VP_ERR_ARG, "bad association sizes");
  if ((q->n_prompt && !q->prompt) || (q->n_copy && !q->copy) || (q->n_nb && (!q->nb_score || !q->nb_seq_off ||
      !q->nb_seq || !q->nb_key_off || !q->nb_keys || !q->nb_pos)) ||
      (q->n_as && (!q->as_tok || !q->as_max || !q->as_cnt)) || (q->n_as_cand && !q->as_cand))
    return dfail(VP_ERR_ARG, "null request array");
  const int nseq = q->n_nb ? q->nb_seq_off[q->n_nb] : 0, nkey = q->n_nb ? q->nb_key_off[q->n_nb] : 0;
  if (nseq < 0 || nkey < 0) return dfail(VP_ERR_ARG, "bad neighbour offsets");
  // one device block: 8-byte arrays first, then the 4-byte ones
  struct Part { const void* src; size_t bytes; size_t off; };
  std::vector<Part> parts = {
      {q->nb_score, 8ull * q->n_nb, 0}, {q->nb_keys, 8ull * nkey, 0}, {q->as_max, 8ull * q->n_as, 0},
      {q->prompt, 4ull * q->n_prompt, 0}, {q->copy, 4ull * q->n_copy, 0},
      {q->nb_seq_off, q->n_nb ? 4ull * (q->n_nb + 1) : 0, 0}, {q->nb_seq, 4ull * nseq, 0},
      {q->nb_key_off, q->n_nb ? 4ull * (q->n_nb + 1) : 0, 0}, {q->nb_pos, 4ull * nkey, 0},
      {q->as_tok, 4ull * q->n_as, 0}, {q->as_cnt, 4ull * q->n_as, 0}, {q->as_cand, 4ull * q->n_as_cand, 0}};
  size_t total = 0;
  for (Part& pt : parts) { pt.off = total; total += (pt.bytes + 15) & ~size_t(15); }
  VD_CUDA(cudaSetDevice(d->device));
  if (total > d->req_cap) {
    if (d->req_buf) cudaFree(d->req_buf);
    d->req_buf = nullptr;
    d->req_cap = 0;
    VD_CUDA(cudaMalloc(&d->req_buf, total ? total : 16));
    d->req_cap = total;
  }
  std::vector<uint8_t> host(total, 0);
  for (const Part& pt : parts)
    if (pt.bytes) std::memcpy(host.data() + pt.off, pt.src, pt.bytes);
  if (total) VD_CUDA(cudaMemcpy(d->req_buf, host.data(), total, cudaMemcpyHostToDevice));
  uint8_t* base = static_cast<uint8_t*>(d->req_buf);
  DraftReq& R = d->req;
  R.nb_score = reinterpret_cast<const double*>(base + parts[0].off);
  R.nb_keys = reinterpret_cast<const unsigned long long*>(base + parts[1].off);
  R.as_max = reinterpret_cast<const double*>(base + parts[2].off);
  R.P = reinterpret_cast<const int32_t*>(base + parts[3].off);
  R.copy = reinterpret_cast<const int32_t*>(base + parts[4].off);
  R.nb_seq_off = reinterpret_cast<const int32_t*>(base + parts[5].off);
  R.nb_seq = reinterpret_cast<const int32_t*>(base + parts[6].off);
  R.nb_key_off = reinterpret_cast<const int32_t*>(base + parts[7].off);
  R.nb_pos = reinterpret_cast<const int32_t*>(base + parts[8].off);
  R.as_tok = reinterpret_cast<const int32_t*>(base + parts[9].off);
  R.as_cnt = reinterpret_cast<const int32_t*>(base + parts[10].off);
  R.as_cand = reinterpret_cast<const int32_t*>(base + parts[11].off);
  R.np = q->n_prompt;
  R.ncopy = q->n_copy;
  R.nnb = q->n_nb;
  R.nas = q->n_as;
  R.nascand = q->n_as_cand;
  d->have_req = true;
  ++d->gen;
  return VP_OK;
}

int vp_draft(vp_drafter* d, const int32_t* d_out_tokens, const vp_state* d_state, int32_t n_out, int32_t B,
             int32_t branch, int32_t* d_tree, const vp_draft_debug* dbg, void* stream) {
  if (!d || !d_tree || (!d_out_tokens && (d_state || n_out > 0))) return dfail(VP_ERR_ARG, "null argument");
  if (!d->have_req) return dfail(VP_ERR_STATE, "vp_drafter_begin first");
  if (B < 0 || B > VP_MAX_ROWS - 1 || branch < 1 || branch > 8) return dfail(VP_ERR_ARG, "B must be 0..15, branch 1..8");
  if (!d_state && n_out < 0) return dfail(VP_ERR_ARG, "negative output length");
  VD_CUDA(cudaSetDevice(d->device));
  DraftOut o = {};
  o.tree = d_tree;
  if (dbg) {
    o.parents = dbg->parents;
    o.tokens = dbg->tokens;
    o.exp_tok = dbg->exp_tokens;
    o.exp_p = dbg->exp_probs;
    o.status = dbg->status;
  }
  k_draft<<<1, DR_THREADS, sizeof(DrShared), static_cast<cudaStream_t>(stream)>>>(
      d->tab, d->req, d_out_tokens, d_state, n_out, B, branch, o);
  VD_CUDA(cudaGetLastError());
  return VP_OK;
}

// ---- CUDA graphs ----

}  // extern "C"

namespace {
// Captures what `enqueue` puts on a private stream and instantiates it.
template <typename F>
int capture(int device, F enqueue, cudaGraphExec_t* out) {
  *out = nullptr;
  VD_CUDA(cudaSetDevice(device));
  cudaStream_t st = nullptr;
  VD_CUDA(cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking));
  cudaGraph_t g = nullptr;
  cudaError_t e = cudaStreamBeginCapture(st, cudaStreamCaptureModeThreadLocal);
  int r = VP_OK;
  if (e == cudaSuccess) {
    r = enqueue(st);
    const cudaError_t e2 = cudaStreamEndCapture(st, &g);  // ends the capture whatever enqueue did
    if (r == VP_OK) e = e2;
  }
  if (r == VP_OK && e == cudaSuccess) e = cudaGraphInstantiate(out, g, 0);
  if (g) cudaGraphDestroy(g);
  cudaStreamDestroy(st);
  if (r != VP_OK) return r;
  if (e != cudaSuccess) {
    *out = nullptr;
    return dfail(VP_ERR_CUDA, std::string("graph capture: ") + cudaGetErrorString(e));
  }
  return VP_OK;
}
}  // namespace

extern "C" {

int vp_pass_graph(vp_ctx* ctx, const int32_t* d_tree, vp_graph** out) {
  if (!ctx || !d_tree || !out) return dfail(VP_ERR_ARG, "null argument");
  *out = nullptr;
  cudaPointerAttributes pa{};
  if (cudaPointerGetAttributes(&pa, d_tree) != cudaSuccess || pa.type != cudaMemoryTypeDevice) {
    cudaGetLastError();
    return dfail(VP_ERR_ARG, "the tree of a pass graph must be device memory");
  }
  vp_graph* g = new vp_graph();
  g->device = pa.device;
  const int r = capture(pa.device, [&](cudaStream_t st) { return vp_pass(ctx, d_tree, st); }, &g->exec);
  if (r != VP_OK) { delete g; return r; }
  *out = g;
  return VP_OK;
}

int vp_step_graph(vp_ctx* ctx, vp_drafter* d, int32_t B, int32_t branch, vp_graph** out) {
  if (!ctx || !d || !out) return dfail(VP_ERR_ARG, "null argument");
  *out = nullptr;
  if (!d->have_req) return dfail(VP_ERR_STATE, "vp_drafter_begin first");
  void* tree = nullptr;
  size_t bytes = 0;
  int r = vp_buffer(ctx, 7, &tree, &bytes);
  if (r) return r;
  const int32_t* toks = vp_device_tokens(ctx);
  const vp_state* st_dev = vp_device_state(ctx);
  if (!toks || !st_dev) return dfail(VP_ERR_ARG, "context without device buffers");
  vp_graph* g = new vp_graph();
  g->device = d->device;
  g->d = d;
  g->gen = d->gen;
  r = capture(d->device, [&](cudaStream_t st) {
    const int rd = vp_draft(d, toks, st_dev, -1, B, branch, static_cast<int32_t*>(tree), nullptr, st);
    return rd ? rd : vp_pass(ctx, static_cast<const int32_t*>(tree), st);
  }, &g->exec);
  if (r != VP_OK) { delete g; return r; }
  *out = g;
  return VP_OK;
}

int vp_graph_launch(vp_graph* g, void* stream) {
  if (!g || !g->exec) return dfail(VP_ERR_ARG, "null graph");
  if (g->d && g->d->gen != g->gen) return dfail(VP_ERR_STATE, "the drafter began another request: capture again");
  VD_CUDA(cudaSetDevice(g->device));
  VD_CUDA(cudaGraphLaunch(g->exec, static_cast<cudaStream_t>(stream)));
  return VP_OK;
}

void vp_graph_destroy(vp_graph* g) {
  if (!g) return;
  if (g->exec) {
    cudaSetDevice(g->device);
    cudaGraphExecDestroy(g->exec);
  }
  delete g;
}

#ifdef VP_DRAFT_TRACE
// Per-phase time of the last k_draft launch, ns summed over its expansions (trace builds only).
int vp_draft_trace(unsigned long long* host) {
  return cudaMemcpyFromSymbol(host, vp::g_dr_trace, sizeof(unsigned long long) * 32) == cudaSuccess ? 0 : -1;
}
#endif

}  // extern "C"
