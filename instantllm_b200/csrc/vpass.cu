// C ABI of the verification pass (include/vpass.h): context, weight packing, pass encoder.
//
// The pass encoder replaces Engine.encodeWidePass / encodePrefill / encodeCommitSpec
// (Sources/Engine/Engine.swift:484-601, 171 Metal dispatches per pass): one verify pass (or one
// 16-row prefill chunk) is ONE cooperative launch of the persistent pass kernel k_pass
// (vp_mega.cuh), one CTA per SM, stages separated by grid barriers.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "vp_commit.cuh"
#include "vp_gemm.cuh"
#include "vp_mega.cuh"
#include "vp_sketch.cuh"

using namespace vp;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

}  // namespace

void vp_set_last_error(const std::string& msg) { g_err = msg; }

namespace {

#define VP_CUDA(call)                                                                  \
  do {                                                                                 \
    cudaError_t e_ = (call);                                                           \
    if (e_ != cudaSuccess)                                                             \
      return fail(VP_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));    \
  } while (0)

// Launch geometry of the stand-alone GEMM kernel (k_gemm), used for the full-logits parity helper
// and the allocation-free argmax.
struct StageCfg {
  int nrb, ng, nsplit, cg, cps;
  size_t smem;
  int grid() const { return nsplit * cps; }
};

StageCfg make_stage(int fmt, int rows, int cols, int nsplit) {
  StageCfg c;
  c.nrb = rows / 16;
  c.ng = cols / GS;
  c.nsplit = nsplit;
  const int per_chunk = mk_chunk_groups(fmt);
  const int ngs = (c.ng + nsplit - 1) / nsplit;
  c.cg = per_chunk < ngs ? per_chunk : ngs;
  c.cps = (c.nrb + GEMM_WARPS - 1) / GEMM_WARPS;
  c.smem = gemm_smem_bytes(fmt, c.ng, nsplit, c.cg);
  return c;
}

}  // namespace

struct vp_ctx {
  vp_config cfg{};
  vp_weights w{};
  bool have_w = false;
  Scratch s{};
  std::vector<void*> allocs;
  StageCfg lm{};          // stand-alone lm_head GEMM (parity helper)
  int grid = 0;           // CTAs of the pass kernel (one per SM)
  int max_chunks = 0;
  unsigned long long* bar = nullptr;
  unsigned* exit_ctr = nullptr;
  unsigned* seq = nullptr;  // pass-kernel launches so far (flag epochs)
  unsigned* gate = nullptr;  // [MK_GATES] stage arrival counters of the pass kernel
  float* lm_pval = nullptr;  // [16][grid] per-CTA argmax partials of the last pass
  int* lm_pidx = nullptr;
  unsigned long long* trace = nullptr;  // stage timestamps of the last pass (ns)
  // device: the state (64 B), the tokens of the last commit (16 int32) and the tree, adjacent so
  // that vp_step moves its inputs in one copy and its results (state + tokens) in one copy
  unsigned char* io = nullptr;
  unsigned char* pin = nullptr;  // pinned host staging of vp_step: the io block in, its head out
  // vp_step as one CUDA graph per input form ([0]: tree only, [1]: state and tree), captured on
  // first use on cap_stream; step_direct: capture failed once, launch the three operations instead
  cudaGraphExec_t step_exec[2] = {nullptr, nullptr};
  cudaStream_t cap_stream = nullptr;
  bool step_direct = false;
};

constexpr size_t IO_TOK = 64;                                   // pass-token offset in ctx->io
constexpr size_t IO_TREE = IO_TOK + ROWS * sizeof(int32_t);     // tree offset in ctx->io
constexpr size_t IO_BYTES = IO_TREE + VP_TREE_INTS * sizeof(int32_t);
constexpr size_t PIN_OUT = 512;                                 // result offset in ctx->pin
static_assert(sizeof(vp_state) <= IO_TOK && IO_BYTES <= PIN_OUT, "io layout");

namespace {

template <typename T>
int dalloc(vp_ctx* c, T** p, size_t bytes) {
  void* q = nullptr;
  cudaError_t e = cudaMalloc(&q, bytes < 16 ? 16 : bytes);
  if (e != cudaSuccess) return fail(VP_ERR_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  e = cudaMemset(q, 0, bytes < 16 ? 16 : bytes);
  if (e != cudaSuccess) return fail(VP_ERR_CUDA, std::string("cudaMemset: ") + cudaGetErrorString(e));
  c->allocs.push_back(q);
  *p = static_cast<T*>(q);
  return VP_OK;
}

template <typename Kern, typename... Args>
cudaError_t launch(Kern kernel, int grid, int block, size_t smem, cudaStream_t st, bool coop, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = coop ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <int FMT, int MODE>
cudaError_t gemm_launch(const StageCfg& c, const GemmParams& p, cudaStream_t st) {
  return launch(k_gemm<FMT, MODE>, c.grid(), GEMM_WARPS * 32, c.smem, st, false, p);
}

template <int FMT>
int set_attrs(vp_ctx* c) {
  VP_CUDA(cudaFuncSetAttribute(k_gemm<FMT, MODE_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               (int)c->lm.smem));
  VP_CUDA(cudaFuncSetAttribute(k_pass<FMT>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MK_SMEM));
  VP_CUDA(cudaFuncSetAttribute(k_pass_groups<FMT, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MK_SMEM));
  VP_CUDA(cudaFuncSetAttribute(k_pass_groups<FMT, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)MK_SMEM));
  int per_sm = 0;
  VP_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k_pass<FMT>, MK_THREADS, MK_SMEM));
  if (per_sm < 1) return fail(VP_ERR_CUDA, "pass kernel does not fit on an SM");
  return VP_OK;
}

MegaParams mega_params(vp_ctx* c) {
  MegaParams p = {};
  p.s = c->s;
  p.embed = static_cast<const uint8_t*>(c->w.embed);
  p.final_norm = c->w.final_norm;
  for (int l = 0; l < c->cfg.n_layers; ++l) {
    p.wqkv[l] = static_cast<const uint8_t*>(c->w.wqkv[l]);
    p.bqkv[l] = c->w.bqkv[l];
    p.wo[l] = static_cast<const uint8_t*>(c->w.wo[l]);
    p.wgu[l] = static_cast<const uint8_t*>(c->w.wgu[l]);
    p.wd[l] = static_cast<const uint8_t*>(c->w.wd[l]);
    p.ln1[l] = c->w.ln1[l];
    p.ln2[l] = c->w.ln2[l];
  }
  p.n_layers = c->cfg.n_layers;
  p.nrb_lm = c->cfg.vocab / 16;
  p.max_chunks = c->max_chunks;
  p.bar = c->bar;
  p.exit_ctr = c->exit_ctr;
  p.seq = c->seq;
  p.gate = c->gate;
  p.lm_pval = c->lm_pval;
  p.lm_pidx = c->lm_pidx;
  p.trace = c->trace;
  return p;
}

int launch_pass(vp_ctx* c, const MegaParams& p, cudaStream_t st) {
  switch (c->cfg.format) {
    case VP_FMT_Q4: VP_CUDA(launch(k_pass<VP_FMT_Q4>, c->grid, MK_THREADS, MK_SMEM, st, true, p)); break;
    case VP_FMT_Q8: VP_CUDA(launch(k_pass<VP_FMT_Q8>, c->grid, MK_THREADS, MK_SMEM, st, true, p)); break;
    case VP_FMT_Q8G32: VP_CUDA(launch(k_pass<VP_FMT_Q8G32>, c->grid, MK_THREADS, MK_SMEM, st, true, p)); break;
    default: VP_CUDA(launch(k_pass<VP_FMT_F16>, c->grid, MK_THREADS, MK_SMEM, st, true, p)); break;
  }
  return VP_OK;
}

int launch_commit(vp_ctx* c, cudaStream_t st) {
  CommitParams cp = {};
  cp.pval = c->lm_pval;
  cp.pidx = c->lm_pidx;
  cp.nparts = c->grid;
  cp.s = c->s;
  VP_CUDA(launch(k_commit, 1, COMMIT_THREADS, 0, st, false, cp));
  return VP_OK;
}

// One launch of the batch kernel: bp.groups requests, each on `per` CTAs (the small-group layout
// below 72 CTAs, where QKV has more row-blocks than CTAs).
int launch_groups(int format, int per, const BatchParams& bp, cudaStream_t st) {
  const bool small = per < QKV / 16;
  const int grid = per * bp.groups;
  switch (format) {
    case VP_FMT_Q4:
      VP_CUDA(launch(small ? k_pass_groups<VP_FMT_Q4, true> : k_pass_groups<VP_FMT_Q4, false>, grid, MK_THREADS,
                     MK_SMEM, st, true, bp));
      break;
    case VP_FMT_Q8:
      VP_CUDA(launch(small ? k_pass_groups<VP_FMT_Q8, true> : k_pass_groups<VP_FMT_Q8, false>, grid, MK_THREADS,
                     MK_SMEM, st, true, bp));
      break;
    case VP_FMT_Q8G32:
      VP_CUDA(launch(small ? k_pass_groups<VP_FMT_Q8G32, true> : k_pass_groups<VP_FMT_Q8G32, false>, grid,
                     MK_THREADS, MK_SMEM, st, true, bp));
      break;
    default:
      VP_CUDA(launch(small ? k_pass_groups<VP_FMT_F16, true> : k_pass_groups<VP_FMT_F16, false>, grid, MK_THREADS,
                     MK_SMEM, st, true, bp));
      break;
  }
  return VP_OK;
}

// Whether a pass fits G CTAs: QKV / O / down take one or two row-blocks per CTA (72 / 56 / 56
// row-blocks), and every CTA keeps its row-blocks' partial tiles of a stage in the MK_PART_SLOTS
// shared-memory slots (QKV and gate/up past the MK_SS_SLOTS of staged RMSNorm partials).
bool split_fits(int G, int vocab) {
  if (G < (QKV / 16 + 1) / 2) return false;
  for (int st = MK_QKV; st <= MK_DOWN; ++st)
    for (int cta = 0; cta < G; ++cta) {
      int rb0, n;
      mk_range(st, cta, G, vocab / 16, rb0, n);
      const int slots = MK_PART_SLOTS - (st == MK_QKV || st == MK_GU ? MK_SS_SLOTS : 0);
      if (n > 2 && st != MK_GU) return false;
      if (n * mk_parts(st, n) > slots) return false;
    }
  return true;
}

int check_ctx(vp_ctx* c) {
  if (!c) return fail(VP_ERR_ARG, "null context");
  if (!c->have_w) return fail(VP_ERR_STATE, "weights not set");
  VP_CUDA(cudaSetDevice(c->cfg.device));
  return VP_OK;
}

}  // namespace

// ------------------------------------------------------------------------------------------------
extern "C" {

const char* vp_last_error(void) { return g_err.c_str(); }

size_t vp_packed_bytes(int32_t format, int32_t rows, int32_t cols) {
  if (rows <= 0 || cols <= 0 || rows % 16 || cols % GS) return 0;
  if (!fmt_valid(format)) return 0;
  return (size_t)(rows / 16) * (cols / GS) * tile_bytes(format);
}

int vp_pack_matrix(int32_t format, int32_t kind, int32_t rows, int32_t cols, const void* d_codes,
                   const void* d_scales, void* d_out, void* stream) {
  if (!vp_packed_bytes(format, rows, cols)) return fail(VP_ERR_ARG, "bad format or shape");
  if (!d_codes || !d_out || (format != VP_FMT_F16 && !d_scales)) return fail(VP_ERR_ARG, "null buffer");
  if (kind == VP_MAT_QKV && (rows != QKV || cols != H)) return fail(VP_ERR_ARG, "QKV must be 1152x896");
  if (kind == VP_MAT_GATEUP && (rows != 2 * F || cols != H)) return fail(VP_ERR_ARG, "gate/up must be 9728x896");
  if (kind < 0 || kind > 2) return fail(VP_ERR_ARG, "bad kind");
  const long long threads = (long long)(rows / 16) * (cols / GS) * 33;
  const int block = 256;
  const int grid = (int)((threads + block - 1) / block);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const uint8_t* cd = static_cast<const uint8_t*>(d_codes);
  const uint8_t* sc = static_cast<const uint8_t*>(d_scales);
  uint8_t* out = static_cast<uint8_t*>(d_out);
  if (format == VP_FMT_Q4) k_pack<VP_FMT_Q4><<<grid, block, 0, st>>>(kind, rows, cols, cd, sc, out);
  else if (format == VP_FMT_Q8) k_pack<VP_FMT_Q8><<<grid, block, 0, st>>>(kind, rows, cols, cd, sc, out);
  else if (format == VP_FMT_Q8G32) k_pack<VP_FMT_Q8G32><<<grid, block, 0, st>>>(kind, rows, cols, cd, sc, out);
  else k_pack<VP_FMT_F16><<<grid, block, 0, st>>>(kind, rows, cols, cd, sc, out);
  VP_CUDA(cudaGetLastError());
  return VP_OK;
}

int vp_create(const vp_config* cfg, vp_ctx** out) {
  if (!cfg || !out) return fail(VP_ERR_ARG, "null argument");
  *out = nullptr;
  if (!fmt_valid(cfg->format)) return fail(VP_ERR_ARG, "format must be q4, q8, q8g32 or f16");
  if (cfg->n_layers < 1 || cfg->n_layers > VP_MAX_LAYERS) return fail(VP_ERR_ARG, "n_layers out of range");
  if (cfg->vocab < 16 || cfg->vocab % 16) return fail(VP_ERR_ARG, "vocab must be a positive multiple of 16");
  if (cfg->vocab > (1 << 24)) return fail(VP_ERR_ARG, "vocab above 2^24");
  if (cfg->max_ctx < ROWS || cfg->max_ctx > (1 << 20)) return fail(VP_ERR_ARG, "max_ctx out of range");
  if (cfg->max_steps < 1 || cfg->max_steps > (1 << 24)) return fail(VP_ERR_ARG, "max_steps out of range");
  VP_CUDA(cudaSetDevice(cfg->device));
  int sms = 0;
  VP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, cfg->device));
  if (!split_fits(sms, cfg->vocab)) return fail(VP_ERR_DEVICE, "the pass kernel needs at least 36 SMs");
  vp_ctx* c = new vp_ctx();
  c->cfg = *cfg;
  const int fmt = cfg->format;
  c->lm = make_stage(fmt, cfg->vocab, H, 1);
  c->lm.cps = std::min(296, (c->lm.nrb + GEMM_WARPS - 1) / GEMM_WARPS);  // two CTAs per SM
  c->max_chunks = (cfg->max_ctx + ATT_SUB - 1) / ATT_SUB + 1;
  c->grid = sms;

  Scratch& s = c->s;
  s.max_ctx = cfg->max_ctx;
  s.max_steps = cfg->max_steps;
  s.vocab = cfg->vocab;
  s.n_layers = cfg->n_layers;
  const size_t kv = (size_t)cfg->n_layers * NKV * cfg->max_ctx * HD * sizeof(__half);
  int r = VP_OK;
  if ((r = dalloc(c, &c->io, IO_BYTES)) || (r = dalloc(c, &s.ri, sizeof(RowInfo))) ||
      (r = dalloc(c, &s.out_tokens, (size_t)cfg->max_steps * sizeof(int32_t))) ||
      (r = dalloc(c, &s.x, ROWS * H * sizeof(float))) || (r = dalloc(c, &s.q, ROWS * H * sizeof(float))) ||
      (r = dalloc(c, &s.act_h, ROWS * H * sizeof(__half))) ||
      (r = dalloc(c, &s.act_f, ROWS * F * sizeof(__half))) ||
      (r = dalloc(c, &s.ss, HRB * ROWS * sizeof(float))) ||
      (r = dalloc(c, &s.part, 256 * sizeof(float))) ||
      (r = dalloc(c, &s.tickets, 2048 * sizeof(int))) ||
      (r = dalloc(c, &s.att_part, (size_t)ROWS * NKV * c->max_chunks * ATT_REC * sizeof(float))) ||
      (r = dalloc(c, &s.kc, kv)) || (r = dalloc(c, &s.vc, kv)) ||
      (r = dalloc(c, &s.rope, (size_t)(cfg->max_ctx + ROWS) * 32 * sizeof(float2))) ||
      (r = dalloc(c, &s.pval, (size_t)ROWS * (cfg->vocab / 16) * sizeof(float))) ||
      (r = dalloc(c, &s.pidx, (size_t)ROWS * (cfg->vocab / 16) * sizeof(int))) ||
      (r = dalloc(c, &c->bar, sizeof(unsigned long long))) ||
      (r = dalloc(c, &c->exit_ctr, sizeof(unsigned))) ||
      (r = dalloc(c, &c->seq, sizeof(unsigned))) ||
      (r = dalloc(c, &s.act_ll, (size_t)H * ROWS / 2 * sizeof(uint64_t))) ||
      (r = dalloc(c, &s.ss_ll, (size_t)HRB * ROWS * sizeof(uint64_t))) ||
      (r = dalloc(c, &s.q_ll, (size_t)ROWS * H * sizeof(uint64_t))) ||
      (r = dalloc(c, &s.kv_ll, (size_t)2 * NKV * ROWS * (HD / 2) * sizeof(uint64_t))) ||
      (r = dalloc(c, &s.att_ll, (size_t)H * ROWS / 2 * sizeof(uint64_t))) ||
      (r = dalloc(c, &s.dn_ll, (size_t)H * ROWS / 2 * sizeof(uint64_t))) ||
      (r = dalloc(c, &s.dn_ss_ll, (size_t)HRB * ROWS * sizeof(uint64_t))) ||
      (r = dalloc(c, &s.dnp_ll, (size_t)HRB * 256 * sizeof(uint64_t))) ||
      (r = dalloc(c, &c->gate, MK_GATES * sizeof(unsigned))) ||
      (r = dalloc(c, &c->lm_pval, (size_t)ROWS * sms * sizeof(float))) ||
      (r = dalloc(c, &c->lm_pidx, (size_t)ROWS * sms * sizeof(int))) ||
      (r = dalloc(c, &c->trace, MK_TRACE * sizeof(unsigned long long)))) {
    vp_destroy(c);
    return r;
  }
  s.st = reinterpret_cast<vp_state*>(c->io);
  s.pass_tok = reinterpret_cast<int32_t*>(c->io + IO_TOK);
  s.tree = reinterpret_cast<int32_t*>(c->io + IO_TREE);
  {
    cudaError_t e = cudaHostAlloc(&c->pin, PIN_OUT + IO_TREE, cudaHostAllocDefault);
    if (e != cudaSuccess) {
      c->pin = nullptr;
      vp_destroy(c);
      return fail(VP_ERR_NOMEM, std::string("cudaHostAlloc: ") + cudaGetErrorString(e));
    }
  }
  // RoPE table: angle = position * theta^(-2i/64) in double, cos/sin rounded once to fp32
  // (tools/reference/qwen_ref.py:107-116).
  {
    std::vector<float2> tab((size_t)(cfg->max_ctx + ROWS) * 32);
    for (int p = 0; p < cfg->max_ctx + ROWS; ++p)
      for (int i = 0; i < 32; ++i) {
        const double inv = 1.0 / std::pow(1000000.0, (double)(2 * i) / 64.0);
        const double a = (double)p * inv;
        tab[(size_t)p * 32 + i] = make_float2((float)std::cos(a), (float)std::sin(a));
      }
    cudaError_t e = cudaMemcpy(s.rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) { vp_destroy(c); return fail(VP_ERR_CUDA, cudaGetErrorString(e)); }
  }
  if (fmt == VP_FMT_Q4) r = set_attrs<VP_FMT_Q4>(c);
  else if (fmt == VP_FMT_Q8) r = set_attrs<VP_FMT_Q8>(c);
  else if (fmt == VP_FMT_Q8G32) r = set_attrs<VP_FMT_Q8G32>(c);
  else r = set_attrs<VP_FMT_F16>(c);
  if (r) { vp_destroy(c); return r; }
  *out = c;
  return VP_OK;
}

void vp_destroy(vp_ctx* c) {
  if (!c) return;
  cudaSetDevice(c->cfg.device);
  for (cudaGraphExec_t& g : c->step_exec)
    if (g) cudaGraphExecDestroy(g);
  if (c->cap_stream) cudaStreamDestroy(c->cap_stream);
  for (void* p : c->allocs) cudaFree(p);
  if (c->pin) cudaFreeHost(c->pin);
  delete c;
}

int vp_set_weights(vp_ctx* c, const vp_weights* w) {
  if (!c || !w) return fail(VP_ERR_ARG, "null argument");
  if (!w->embed || !w->final_norm) return fail(VP_ERR_ARG, "embed / final_norm missing");
  for (int l = 0; l < c->cfg.n_layers; ++l)
    if (!w->wqkv[l] || !w->bqkv[l] || !w->wo[l] || !w->wgu[l] || !w->wd[l] || !w->ln1[l] || !w->ln2[l])
      return fail(VP_ERR_ARG, "layer weight missing");
  c->w = *w;
  c->have_w = true;
  for (cudaGraphExec_t& g : c->step_exec)  // they hold the previous weights' pointers
    if (g) {
      cudaGraphExecDestroy(g);
      g = nullptr;
    }
  return VP_OK;
}

size_t vp_prefix_bytes(vp_ctx* c, int32_t n) {
  if (!c || n < 1 || n > c->cfg.max_ctx) return 0;
  return (size_t)2 * c->cfg.n_layers * NKV * n * HD * sizeof(__half);
}

// Copies the first n rows of every (layer, kv head) slab of the K and V caches to or from the host:
// one strided 2-D copy per cache (slab pitch max_ctx rows, n rows each).
static int prefix_copy(vp_ctx* c, int32_t n, void* host, bool save, cudaStream_t st) {
  const size_t row = (size_t)HD * sizeof(__half), slabs = (size_t)c->cfg.n_layers * NKV;
  const size_t dev_pitch = (size_t)c->cfg.max_ctx * row, host_pitch = (size_t)n * row;
  for (int which = 0; which < 2; ++which) {
    __half* dev = which ? c->s.vc : c->s.kc;
    uint8_t* h = static_cast<uint8_t*>(host) + (size_t)which * slabs * host_pitch;
    if (save)
      VP_CUDA(cudaMemcpy2DAsync(h, host_pitch, dev, dev_pitch, host_pitch, slabs, cudaMemcpyDeviceToHost, st));
    else
      VP_CUDA(cudaMemcpy2DAsync(dev, dev_pitch, h, host_pitch, host_pitch, slabs, cudaMemcpyHostToDevice, st));
  }
  return VP_OK;
}

int vp_save_prefix(vp_ctx* c, int32_t n, void* host, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  if (!host || !vp_prefix_bytes(c, n)) return fail(VP_ERR_ARG, "bad prefix length or buffer");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if ((r = prefix_copy(c, n, host, true, st))) return r;
  VP_CUDA(cudaStreamSynchronize(st));
  return VP_OK;
}

int vp_load_prefix(vp_ctx* c, int32_t n, const void* host, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  if (!host || !vp_prefix_bytes(c, n) || n + ROWS > c->cfg.max_ctx) return fail(VP_ERR_ARG, "bad prefix length or buffer");
  return prefix_copy(c, n, const_cast<void*>(host), false, static_cast<cudaStream_t>(stream));
}

int vp_begin(vp_ctx* c, int32_t cached, int32_t max_new, int32_t eos0, int32_t eos1, void* stream) {
  if (!c) return fail(VP_ERR_ARG, "null context");
  if (cached < 0 || max_new < 1 || max_new > c->cfg.max_steps) return fail(VP_ERR_ARG, "bad request size");
  if (cached + max_new + ROWS > c->cfg.max_ctx) return fail(VP_ERR_ARG, "request exceeds max_ctx");
  VP_CUDA(cudaSetDevice(c->cfg.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  k_begin<<<64, 256, 0, st>>>(c->s.st, c->s.out_tokens, c->cfg.max_steps, (int)cached, (int)max_new,
                              (int)eos0, (int)eos1, c->cfg.max_ctx, 0);
  VP_CUDA(cudaGetLastError());
  return VP_OK;
}

int vp_prefill(vp_ctx* c, const int32_t* d_tokens, int32_t n, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  if (!d_tokens || n < 1) return fail(VP_ERR_ARG, "empty prompt");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int c0 = 0; c0 < n; c0 += ROWS) {
    const int cn = n - c0 < ROWS ? n - c0 : ROWS;
    const bool last = c0 + cn == n;
    MegaParams p = mega_params(c);
    p.prompt = d_tokens + c0;
    p.chunk_n = cn;
    p.chunk_start = c0;
    p.total_n = n;
    p.do_lm = last;
    p.do_commit = last;
    if ((r = launch_pass(c, p, st))) return r;
  }
  return VP_OK;
}

int vp_verify(vp_ctx* c, const int32_t* tree, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  if (!tree) return fail(VP_ERR_ARG, "null tree");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  VP_CUDA(cudaMemcpyAsync(c->s.tree, tree, VP_TREE_INTS * sizeof(int32_t), cudaMemcpyDefault, st));
  MegaParams p = mega_params(c);
  p.do_lm = 1;
  return launch_pass(c, p, st);
}

int vp_verify_chain(vp_ctx* c, const int32_t* drafts, int32_t nd, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  if (nd < 0 || nd > ROWS - 1 || (nd > 0 && !drafts)) return fail(VP_ERR_ARG, "bad draft count");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  k_chain_tree<<<1, 32, 0, st>>>(c->s.tree, drafts, nd);
  VP_CUDA(cudaGetLastError());
  MegaParams p = mega_params(c);
  p.do_lm = 1;
  return launch_pass(c, p, st);
}

int vp_commit(vp_ctx* c, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  return launch_commit(c, static_cast<cudaStream_t>(stream));
}

int vp_pass(vp_ctx* c, const int32_t* tree, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  if (!tree) return fail(VP_ERR_ARG, "null tree");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (tree != c->s.tree)  // a drafter may have written the context's own tree buffer (vp_buffer 7)
    VP_CUDA(cudaMemcpyAsync(c->s.tree, tree, VP_TREE_INTS * sizeof(int32_t), cudaMemcpyDefault, st));
  MegaParams p = mega_params(c);
  p.do_lm = 1;
  p.do_commit = 1;
  return launch_pass(c, p, st);
}

int vp_pass_batch(vp_ctx* const* ctxs, const int32_t* const* trees, int32_t n, int32_t shares, void* stream) {
  if (!ctxs || !trees || shares < 1 || shares > MK_MAX_GROUPS || n < 1 || n > shares)
    return fail(VP_ERR_ARG, "need 1 <= n <= shares <= 4");
  int r = VP_OK;
  for (int i = 0; i < n; ++i) {
    if ((r = check_ctx(ctxs[i]))) return r;
    if (!trees[i]) return fail(VP_ERR_ARG, "null tree");
    for (int j = 0; j < i; ++j)
      if (ctxs[j] == ctxs[i]) return fail(VP_ERR_ARG, "the same context twice");
    if (ctxs[i]->cfg.device != ctxs[0]->cfg.device || ctxs[i]->cfg.format != ctxs[0]->cfg.format)
      return fail(VP_ERR_ARG, "contexts on different devices or formats");
  }
  vp_ctx* c0 = ctxs[0];
  const int per = c0->grid / shares;  // every request gets its share, whatever n is
  for (int i = 0; i < n; ++i)
    if (!split_fits(per, ctxs[i]->cfg.vocab)) return fail(VP_ERR_DEVICE, "too few SMs for that many pass groups");
  VP_CUDA(cudaSetDevice(c0->cfg.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  BatchParams bp = {};
  bp.groups = n;
  for (int i = 0; i < n; ++i) {
    if (trees[i] != ctxs[i]->s.tree)  // a drafter that wrote the context's own tree buffer: no copy
      VP_CUDA(cudaMemcpyAsync(ctxs[i]->s.tree, trees[i], VP_TREE_INTS * sizeof(int32_t), cudaMemcpyDefault, st));
    bp.p[i] = mega_params(ctxs[i]);
    bp.p[i].do_lm = 1;
    bp.p[i].do_commit = 1;
  }
  return launch_groups(c0->cfg.format, per, bp, st);
}

int vp_prefill_batch(vp_ctx* const* ctxs, const int32_t* const* d_tokens, const int32_t* n, int32_t k,
                     int32_t shares, void* stream) {
  if (!ctxs || !d_tokens || !n || shares < 1 || shares > MK_MAX_GROUPS || k < 1 || k > shares)
    return fail(VP_ERR_ARG, "need 1 <= k <= shares <= 4");
  int r = VP_OK, longest = 0;
  for (int i = 0; i < k; ++i) {
    if ((r = check_ctx(ctxs[i]))) return r;
    if (!d_tokens[i] || n[i] < 1) return fail(VP_ERR_ARG, "empty prompt");
    for (int j = 0; j < i; ++j)
      if (ctxs[j] == ctxs[i]) return fail(VP_ERR_ARG, "the same context twice");
    if (ctxs[i]->cfg.device != ctxs[0]->cfg.device || ctxs[i]->cfg.format != ctxs[0]->cfg.format)
      return fail(VP_ERR_ARG, "contexts on different devices or formats");
    longest = std::max(longest, (int)n[i]);
  }
  vp_ctx* c0 = ctxs[0];
  const int per = c0->grid / shares;
  for (int i = 0; i < k; ++i)
    if (!split_fits(per, ctxs[i]->cfg.vocab)) return fail(VP_ERR_DEVICE, "too few SMs for that many pass groups");
  VP_CUDA(cudaSetDevice(c0->cfg.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // chunk c of every request whose prompt has one, the requests of a launch on their shares
  for (int c = 0; c < longest; c += ROWS) {
    BatchParams bp = {};
    for (int i = 0; i < k; ++i) {
      if (c >= n[i]) continue;
      const int cn = n[i] - c < ROWS ? n[i] - c : ROWS;
      const bool last = c + cn == n[i];
      MegaParams& p = bp.p[bp.groups++];
      p = mega_params(ctxs[i]);
      p.prompt = d_tokens[i] + c;
      p.chunk_n = cn;
      p.chunk_start = c;
      p.total_n = n[i];
      p.do_lm = last;
      p.do_commit = last;
    }
    if ((r = launch_groups(c0->cfg.format, per, bp, st))) return r;
  }
  return VP_OK;
}

int vp_pass_multi(vp_ctx* const* ctxs, const int32_t* const* trees, int32_t n, void* stream) {
  if (n < 1 || n > 2) return fail(VP_ERR_ARG, "n must be 1 or 2");
  return vp_pass_batch(ctxs, trees, n, 2, stream);
}

namespace {
// vp_step's operations on ctx c: the io block in from the pinned staging block (from byte `off`),
// the pass, the state and the pass's tokens out to the staging block.
int step_ops(vp_ctx* c, size_t off, cudaStream_t st) {
  VP_CUDA(cudaMemcpyAsync(c->io + off, c->pin + off, IO_BYTES - off, cudaMemcpyHostToDevice, st));
  MegaParams p = mega_params(c);
  p.do_lm = 1;
  p.do_commit = 1;
  const int r = launch_pass(c, p, st);
  if (r) return r;
  VP_CUDA(cudaMemcpyAsync(c->pin + PIN_OUT, c->io, IO_TREE, cudaMemcpyDeviceToHost, st));
  return VP_OK;
}

// The graph of step_ops for one input form, captured once (a thread-local capture on a stream of
// the context's own): every later vp_step is one graph launch instead of three operations.
cudaGraphExec_t step_graph(vp_ctx* c, int with_state) {
  if (c->step_exec[with_state] || c->step_direct) return c->step_exec[with_state];
  bool ok = cudaSetDevice(c->cfg.device) == cudaSuccess;
  if (ok && !c->cap_stream) ok = cudaStreamCreateWithFlags(&c->cap_stream, cudaStreamNonBlocking) == cudaSuccess;
  cudaGraph_t g = nullptr;
  if (ok) ok = cudaStreamBeginCapture(c->cap_stream, cudaStreamCaptureModeThreadLocal) == cudaSuccess;
  if (ok) {
    const int r = step_ops(c, with_state ? 0 : IO_TOK, c->cap_stream);
    ok = cudaStreamEndCapture(c->cap_stream, &g) == cudaSuccess && r == VP_OK && g;
  }
  if (ok) ok = cudaGraphInstantiate(&c->step_exec[with_state], g, 0) == cudaSuccess;
  if (g) cudaGraphDestroy(g);
  if (!ok) {
    cudaGetLastError();  // a failed capture leaves no error behind: vp_step launches directly
    c->step_exec[with_state] = nullptr;
    c->step_direct = true;
  }
  return c->step_exec[with_state];
}
}  // namespace

int vp_step(vp_ctx* c, const vp_state* state_in, const int32_t* tree, vp_state* state_out,
            int32_t* tokens_out, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  if (!tree || !state_out) return fail(VP_ERR_ARG, "null tree or state_out");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The previous call synchronised this stream (also on its error paths), so the staging block is
  // free to reuse.
  std::memcpy(c->pin + IO_TREE, tree, VP_TREE_INTS * sizeof(int32_t));
  // no tokens unless the commit runs (a finished or failed request skips it)
  std::memset(c->pin + IO_TOK, 0xff, IO_TREE - IO_TOK);
  if (state_in) std::memcpy(c->pin, state_in, sizeof(vp_state));
  const cudaGraphExec_t g = step_graph(c, state_in ? 1 : 0);
  if (g) {
    const cudaError_t e = cudaGraphLaunch(g, st);
    if (e != cudaSuccess) r = fail(VP_ERR_CUDA, std::string("cudaGraphLaunch: ") + cudaGetErrorString(e));
  } else {
    r = step_ops(c, state_in ? 0 : IO_TOK, st);
  }
  const cudaError_t se = cudaStreamSynchronize(st);  // also on failure: the staging block is in use
  if (r) return r;
  if (se != cudaSuccess) return fail(VP_ERR_CUDA, std::string("cudaStreamSynchronize: ") + cudaGetErrorString(se));
  std::memcpy(state_out, c->pin + PIN_OUT, sizeof(vp_state));
  if (tokens_out) std::memcpy(tokens_out, c->pin + PIN_OUT + IO_TOK, ROWS * sizeof(int32_t));
  return state_out->err ? VP_ERR_DEVICE : VP_OK;
}

int vp_read_state(vp_ctx* c, vp_state* host, void* stream) {
  if (!c || !host) return fail(VP_ERR_ARG, "null argument");
  VP_CUDA(cudaSetDevice(c->cfg.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  VP_CUDA(cudaMemcpyAsync(host, c->s.st, sizeof(vp_state), cudaMemcpyDeviceToHost, st));
  VP_CUDA(cudaStreamSynchronize(st));
  return host->err ? VP_ERR_DEVICE : VP_OK;
}

int vp_write_state(vp_ctx* c, const vp_state* state, int32_t from_device, void* stream) {
  if (!c || !state) return fail(VP_ERR_ARG, "null argument");
  VP_CUDA(cudaSetDevice(c->cfg.device));
  VP_CUDA(cudaMemcpyAsync(c->s.st, state, sizeof(vp_state),
                          from_device ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice,
                          static_cast<cudaStream_t>(stream)));
  return VP_OK;
}

int vp_read_tokens(vp_ctx* c, int32_t* host, int32_t count, void* stream) {
  if (!c || !host || count < 0 || count > c->cfg.max_steps) return fail(VP_ERR_ARG, "bad argument");
  VP_CUDA(cudaSetDevice(c->cfg.device));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  VP_CUDA(cudaMemcpyAsync(host, c->s.out_tokens, count * sizeof(int32_t), cudaMemcpyDeviceToHost, st));
  VP_CUDA(cudaStreamSynchronize(st));
  return VP_OK;
}

int32_t* vp_device_tokens(vp_ctx* c) { return c ? c->s.out_tokens : nullptr; }
vp_state* vp_device_state(vp_ctx* c) { return c ? c->s.st : nullptr; }

int vp_debug_logits(vp_ctx* c, float* d_out, void* stream) {
  int r = check_ctx(c);
  if (r) return r;
  if (!d_out) return fail(VP_ERR_ARG, "null output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  GemmParams p = {};
  p.w = static_cast<const uint8_t*>(c->w.embed);
  p.act = c->s.act_h;
  p.nrb = c->lm.nrb;
  p.ng = c->lm.ng;
  p.nsplit = 1;
  p.cg = c->lm.cg;
  p.cps = c->lm.cps;
  p.s = c->s;
  p.ss_in = c->s.ss;
  p.pval = c->s.pval;
  p.pidx = c->s.pidx;
  p.dbg = d_out;
  switch (c->cfg.format) {
    case VP_FMT_Q4: VP_CUDA((gemm_launch<VP_FMT_Q4, MODE_ARGMAX>(c->lm, p, st))); break;
    case VP_FMT_Q8: VP_CUDA((gemm_launch<VP_FMT_Q8, MODE_ARGMAX>(c->lm, p, st))); break;
    case VP_FMT_Q8G32: VP_CUDA((gemm_launch<VP_FMT_Q8G32, MODE_ARGMAX>(c->lm, p, st))); break;
    default: VP_CUDA((gemm_launch<VP_FMT_F16, MODE_ARGMAX>(c->lm, p, st))); break;
  }
  return VP_OK;
}

int vp_buffer(vp_ctx* c, int32_t which, void** ptr, size_t* bytes) {
  if (!c || !ptr || !bytes) return fail(VP_ERR_ARG, "null argument");
  const size_t kv = (size_t)c->cfg.n_layers * NKV * c->cfg.max_ctx * HD * sizeof(__half);
  const size_t pv = (size_t)ROWS * c->grid * 4;
  switch (which) {
    case 0: *ptr = c->s.x; *bytes = ROWS * H * 4; break;
    case 1: *ptr = c->s.q; *bytes = ROWS * H * 4; break;
    case 2: *ptr = c->s.kc; *bytes = kv; break;
    case 3: *ptr = c->s.vc; *bytes = kv; break;
    case 4: *ptr = c->lm_pval; *bytes = pv; break;
    case 5: *ptr = c->lm_pidx; *bytes = pv; break;
    case 6: *ptr = c->trace; *bytes = MK_TRACE * sizeof(unsigned long long); break;
    case 7: *ptr = c->s.tree; *bytes = VP_TREE_INTS * sizeof(int32_t); break;
    default: return fail(VP_ERR_ARG, "unknown buffer");
  }
  return VP_OK;
}

}  // extern "C"

// ------------------------------------------------------------------------------------------------
// Greedy lm-head argmax that allocates nothing (vp_head_argmax_noalloc).
//
// For callers that cannot call cudaMalloc: its scratch (the fp16 normed rows, the RMSNorm
// partials, a state / row-info block and the per-row argmax keys) is this file-scope
// device array. Host code must never use `g_noalloc_scratch` itself as a pointer: on the host it
// is only a stand-in symbol. The device address is looked up once per device with
// cudaGetSymbolAddress and passed to the kernels.

namespace {

constexpr size_t na_align(size_t v) { return (v + 255) & ~size_t(255); }
constexpr size_t NA_ACT = na_align(ROWS * H * sizeof(__half));
constexpr size_t NA_SS = na_align(HRB * ROWS * sizeof(float));
constexpr size_t NA_ST = na_align(sizeof(vp_state));
constexpr size_t NA_RI = na_align(sizeof(RowInfo));
constexpr size_t NA_KEYS = na_align(sizeof(ArgmaxKeys));
constexpr size_t NA_BYTES = NA_ACT + NA_SS + NA_ST + NA_RI + NA_KEYS;

}  // namespace

static __device__ __align__(256) unsigned char g_noalloc_scratch[NA_BYTES];

namespace {

// x rows -> half(x * final_norm) act blocks and per-row-block sums of squares, with the same
// expressions and reduction order as the residual epilogue that feeds the pass's own lm_head.
__device__ void na_prep_body(const float* x, const float* wnorm, int rows, __half* act, float* ss,
                             vp_state* st, RowInfo* ri) {
  const int rb = blockIdx.x, lane = threadIdx.x, gid = lane >> 2, tid4 = lane & 3;
  const int d0 = rb * 16 + gid, d1 = d0 + 8;
  const float w0 = wnorm[d0], w1 = wnorm[d1];
#pragma unroll
  for (int nt = 0; nt < 2; ++nt)
#pragma unroll
    for (int e = 0; e < 2; ++e) {
      const int t = nt * 8 + 2 * tid4 + e;
      float v0 = 0.f, v1 = 0.f;
      if (t < rows) {
        v0 = x[t * H + d0];
        v1 = x[t * H + d1];
      }
      act[act_index(t, d0)] = __float2half_rn(v0 * w0);
      act[act_index(t, d1)] = __float2half_rn(v1 * w1);
      float sq = v0 * v0 + v1 * v1;
      sq += __shfl_xor_sync(0xffffffffu, sq, 4);
      sq += __shfl_xor_sync(0xffffffffu, sq, 8);
      sq += __shfl_xor_sync(0xffffffffu, sq, 16);
      if (gid == 0) ss[rb * 16 + t] = sq;
    }
  if (rb == 0 && lane == 0) {
    vp_state z = {};
    *st = z;  // the array keeps the previous call's contents: the error bits must start clear
    ri->n = rows;
    ri->pos = 0;
    ri->mode = 0;
    ri->live = 1;
  }
}

__global__ void k_na_prep(const float* x, const float* wnorm, int rows, __half* act, float* ss,
                          vp_state* st, RowInfo* ri, ArgmaxKeys* keys) {
  na_prep_body(x, wnorm, rows, act, ss, st, ri);
  if (blockIdx.x == 1) {
    unsigned* z = reinterpret_cast<unsigned*>(keys);
    for (int i = threadIdx.x; i < (int)(sizeof(ArgmaxKeys) / 4); i += blockDim.x) z[i] = 0u;
  }
}

// The sketch head's first launch: the same normed rows, plus a cleared per-call block.
__global__ void k_sk_prep(const float* x, const float* wnorm, int rows, __half* act, float* ss,
                          vp_state* st, RowInfo* ri, SketchSmall* small) {
  na_prep_body(x, wnorm, rows, act, ss, st, ri);
  if (blockIdx.x == 1) {
    unsigned* z = reinterpret_cast<unsigned*>(small);
    for (int i = threadIdx.x; i < (int)(sizeof(SketchSmall) / 4); i += blockDim.x) z[i] = 0u;
  }
}

// Per-device set-up state. Only a successful look-up is kept: a failed one (for example a first
// call made during stream capture) is retried by the next call.
struct NoAllocDevice {
  std::mutex mu;
  bool ready = false;
  void* base = nullptr;
};
NoAllocDevice g_na_dev[64];

template <int FMT>
cudaError_t na_smem_attr() {
  const size_t need = make_stage(FMT, 16, H, 1).smem;
  cudaFuncAttributes a;
  cudaError_t e = cudaFuncGetAttributes(&a, k_gemm<FMT, MODE_ARGMAX>);
  if (e != cudaSuccess) return e;
  if ((size_t)a.maxDynamicSharedSizeBytes >= need) return cudaSuccess;
  return cudaFuncSetAttribute(k_gemm<FMT, MODE_ARGMAX>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)need);
}

// Once per device, with that device current: the device address of the static scratch array.
int na_setup(int dev, unsigned char** base) {
  NoAllocDevice& d = g_na_dev[dev];
  std::lock_guard<std::mutex> lock(d.mu);
  if (!d.ready) {
    void* b = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&b, g_noalloc_scratch);
    if (e == cudaSuccess) e = na_smem_attr<VP_FMT_Q4>();
    if (e == cudaSuccess) e = na_smem_attr<VP_FMT_Q8>();
    if (e == cudaSuccess) e = na_smem_attr<VP_FMT_Q8G32>();
    if (e == cudaSuccess) e = na_smem_attr<VP_FMT_F16>();
    if (e != cudaSuccess) return fail(VP_ERR_CUDA, std::string("no-alloc set-up: ") + cudaGetErrorString(e));
    d.base = b;
    d.ready = true;
  }
  *base = static_cast<unsigned char*>(d.base);
  return VP_OK;
}

}  // namespace

extern "C" int vp_head_argmax_noalloc(int32_t format, int32_t vocab, const void* d_embed,
                                      const float* d_final_norm, const float* d_x, int32_t rows,
                                      int32_t* d_tokens, void* stream) {
  if (!fmt_valid(format)) return fail(VP_ERR_ARG, "format must be q4, q8, q8g32 or f16");
  if (vocab < 16 || vocab % 16 || vocab > VP_NOALLOC_MAX_VOCAB)
    return fail(VP_ERR_ARG, "vocab must be a multiple of 16 and at most VP_NOALLOC_MAX_VOCAB (163840)");
  if (rows < 1 || rows > ROWS) return fail(VP_ERR_ARG, "rows must be 1..16");
  if (!d_embed || !d_final_norm || !d_x || !d_tokens) return fail(VP_ERR_ARG, "null buffer");
  int dev = 0;
  VP_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(VP_ERR_ARG, "device ordinal above 63");
  unsigned char* base = nullptr;
  int r = na_setup(dev, &base);
  if (r) return r;
  __half* act = reinterpret_cast<__half*>(base);
  float* ss = reinterpret_cast<float*>(base + NA_ACT);
  vp_state* st = reinterpret_cast<vp_state*>(base + NA_ACT + NA_SS);
  RowInfo* ri = reinterpret_cast<RowInfo*>(base + NA_ACT + NA_SS + NA_ST);
  ArgmaxKeys* keys = reinterpret_cast<ArgmaxKeys*>(base + NA_ACT + NA_SS + NA_ST + NA_RI);
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  k_na_prep<<<HRB, 32, 0, s>>>(d_x, d_final_norm, rows, act, ss, st, ri, keys);
  VP_CUDA(cudaGetLastError());
  StageCfg lm = make_stage(format, vocab, H, 1);
  lm.cps = std::min(296, (lm.nrb + GEMM_WARPS - 1) / GEMM_WARPS);  // two CTAs per SM
  GemmParams p = {};
  p.w = static_cast<const uint8_t*>(d_embed);
  p.act = act;
  p.nrb = lm.nrb;
  p.ng = lm.ng;
  p.nsplit = 1;
  p.cg = lm.cg;
  p.cps = lm.cps;
  p.ss_in = ss;
  p.keys = keys;
  p.tokens = d_tokens;
  p.out_rows = rows;
  p.s.st = st;
  p.s.ri = ri;
  switch (format) {
    case VP_FMT_Q4: VP_CUDA((gemm_launch<VP_FMT_Q4, MODE_ARGMAX>(lm, p, s))); break;
    case VP_FMT_Q8: VP_CUDA((gemm_launch<VP_FMT_Q8, MODE_ARGMAX>(lm, p, s))); break;
    case VP_FMT_Q8G32: VP_CUDA((gemm_launch<VP_FMT_Q8G32, MODE_ARGMAX>(lm, p, s))); break;
    default: VP_CUDA((gemm_launch<VP_FMT_F16, MODE_ARGMAX>(lm, p, s))); break;
  }
  return VP_OK;
}

// ------------------------------------------------------------------------------------------------
// Two-stage lm_head over the 2-bit sketch (vp_head_argmax_sketch; kernels in vp_sketch.cuh).

namespace {

struct SkWork {
  __half* act;
  float* ss;
  vp_state* st;
  RowInfo* ri;
  SketchSmall* small;
  float* bounds;
  size_t bounds_off;
  size_t bytes;
};

SkWork sk_work(int vocab, unsigned char* base) {
  const size_t ngrp = sk_groups(vocab);
  size_t o = 0;
  SkWork w;
  auto take = [&](size_t n) { unsigned char* q = base ? base + o : nullptr; o += na_align(n); return q; };
  w.act = reinterpret_cast<__half*>(take(ROWS * H * sizeof(__half)));
  w.ss = reinterpret_cast<float*>(take(HRB * ROWS * sizeof(float)));
  w.st = reinterpret_cast<vp_state*>(take(sizeof(vp_state)));
  w.ri = reinterpret_cast<RowInfo*>(take(sizeof(RowInfo)));
  w.small = reinterpret_cast<SketchSmall*>(take(sizeof(SketchSmall)));
  w.bounds_off = o;
  w.bounds = reinterpret_cast<float*>(take(2 * ROWS * ngrp * sizeof(float)));
  w.bytes = o;
  return w;
}

bool sk_vocab_ok(int vocab) { return vocab >= 16 && vocab % 16 == 0 && vocab <= (1 << 26); }

}  // namespace

extern "C" {

size_t vp_sketch_bytes(int32_t vocab) {
  return sk_vocab_ok(vocab) ? (size_t)(vocab / 16) * SK_NG * SK_TILE : 0;
}

int vp_pack_sketch(int32_t vocab, const void* d_hi, void* d_out, void* stream) {
  if (!sk_vocab_ok(vocab)) return fail(VP_ERR_ARG, "vocab must be a positive multiple of 16");
  if (!d_hi || !d_out) return fail(VP_ERR_ARG, "null buffer");
  const long long n = (long long)(vocab / 16) * SK_NG * 32;
  k_pack_sketch<<<(unsigned)((n + 255) / 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      vocab, static_cast<const uint8_t*>(d_hi), static_cast<uint8_t*>(d_out));
  VP_CUDA(cudaGetLastError());
  return VP_OK;
}

size_t vp_sketch_bounds_offset(void) { return sk_work(32, nullptr).bounds_off; }

size_t vp_sketch_work_bytes(int32_t vocab) {
  return sk_vocab_ok(vocab) ? sk_work(vocab, nullptr).bytes : 0;
}

int vp_head_argmax_sketch(int32_t vocab, const void* d_embed, const void* d_sketch,
                          const float* d_final_norm, const float* d_x, int32_t rows, float k_sigma,
                          void* d_work, size_t work_bytes, int32_t* d_tokens, int32_t* d_ncand,
                          void* stream) {
  if (!sk_vocab_ok(vocab)) return fail(VP_ERR_ARG, "vocab must be a positive multiple of 16");
  if (rows < 1 || rows > ROWS) return fail(VP_ERR_ARG, "rows must be 1..16");
  if (!(k_sigma > 0.f) || !std::isfinite(k_sigma)) return fail(VP_ERR_ARG, "k_sigma must be positive");
  if (!d_embed || !d_sketch || !d_final_norm || !d_x || !d_work || !d_tokens)
    return fail(VP_ERR_ARG, "null buffer");
  if (reinterpret_cast<uintptr_t>(d_work) % 256 || reinterpret_cast<uintptr_t>(d_sketch) % 16 ||
      reinterpret_cast<uintptr_t>(d_embed) % 16)
    return fail(VP_ERR_ARG, "work must be 256-byte aligned, sketch and embed 16-byte aligned");
  const SkWork w = sk_work(vocab, static_cast<unsigned char*>(d_work));
  if (work_bytes < w.bytes) return fail(VP_ERR_ARG, "work buffer smaller than vp_sketch_work_bytes");
  int dev = 0, sms = 0;
  VP_CUDA(cudaGetDevice(&dev));
  VP_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
  cudaStream_t s = static_cast<cudaStream_t>(stream);

  SketchParams p = {};
  p.sk = static_cast<const uint8_t*>(d_sketch);
  p.emb = static_cast<const uint8_t*>(d_embed);
  p.act = w.act;
  p.ss = w.ss;
  p.bounds = w.bounds;
  p.small = w.small;
  p.tokens = d_tokens;
  p.ncand = d_ncand;
  p.nrb = vocab / 16;
  p.ngrp = sk_groups(vocab);
  p.rows = rows;
  p.k = k_sigma;

  k_sk_prep<<<HRB, 32, 0, s>>>(d_x, d_final_norm, rows, w.act, w.ss, w.st, w.ri, w.small);
  VP_CUDA(cudaGetLastError());
  const int g1 = std::min((p.ngrp + SK_WARPS - 1) / SK_WARPS, 2 * sms);  // resident CTAs
  if (rows <= 8) k_sketch<1><<<g1, SK_THREADS, 0, s>>>(p);
  else k_sketch<2><<<g1, SK_THREADS, 0, s>>>(p);
  VP_CUDA(cudaGetLastError());
  // one wave: stage 2 runs one 253-register CTA per SM
  const int g2 = std::min(std::max(sms, (p.ngrp + SK_MAX_GPC - 1) / SK_MAX_GPC), p.ngrp);
  k_sk_exact<<<g2, SK_THREADS, 0, s>>>(p);
  VP_CUDA(cudaGetLastError());
  return VP_OK;
}

}  // extern "C"
