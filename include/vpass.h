/*
 * vpass.h - C ABI of the B200 speculative-decoding verification pass (Qwen2.5-0.5B architecture).
 *
 * The reference engine (instantllm, Swift + Metal) has no FFI layer: its operator surface is the
 * Engine class. Each entry point below names the Engine member or Metal kernel it replaces
 * (paths inside the instantllm project).
 *
 * Conventions
 *  - Every function returns VP_OK (0) or a negative VP_ERR_* code; nothing throws or aborts.
 *  - Pointers named d_* are device pointers (or any pointer cudaMemcpyDefault accepts where noted).
 *    `stream` is a cudaStream_t passed as void* so this header needs no CUDA include.
 *  - Work is stream-ordered. Only vp_read_state synchronises (on the given stream).
 *  - A context owns its scratch (activations, KV cache, partials, state, token buffer). Weights are
 *    borrowed: the caller keeps the packed weight buffers alive (Engine.swift:96-99 borrows the
 *    mmapped model the same way).
 *  - One context serves one request at a time on one GPU and is not thread-safe. Contexts on
 *    different GPUs are independent (request-level sharding needs no communication).
 *  - Device-side failures (bad tree, context overflow, wait timeout) never trap: they set
 *    vp_state.err and vp_state.done, and every later kernel of the request returns at once.
 */
#ifndef VPASS_H
#define VPASS_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Architecture constants (docs/SPEC.md:31-44; tools/reference/qwen_ref.py:40-51). */
#define VP_HIDDEN 896
#define VP_FFN 4864
#define VP_NQ_HEADS 14
#define VP_NKV_HEADS 2
#define VP_HEAD_DIM 64
#define VP_QKV_ROWS 1152
#define VP_MAX_LAYERS 24
#define VP_MAX_ROWS 16 /* rows per verify pass: root + 15 drafts (Shaders.swift:23-30) */
#define VP_GROUP 64    /* quantisation group along K for q4 and q8 */

/* Tree buffer, int32[VP_TREE_INTS] (Shaders.swift:23-30, written by k_ildraft :846-866):
 * [0] n rows; [1+i] depth[i]; [17+i] parent[i]; [33+i] tok[i]; [49+i] ancestor bitmask[i].
 * Row 0 is the last committed token (its tok entry is ignored: the device state supplies it).
 * Row i > 0 is a draft whose parent row parent[i] < i, with depth[i] = depth[parent[i]] + 1.
 * Row i sits at KV slot pos + i and is rotated (RoPE) as position pos + depth[i]. */
#define VP_TREE_INTS 65
#define VP_TR_N 0
#define VP_TR_DEPTH 1
#define VP_TR_PARENT 17
#define VP_TR_TOK 33
#define VP_TR_ANC 49

/* VP_FMT_Q8 is int8 with one scale per 64 columns; VP_FMT_Q8G32 is the
 * reference's own q8 layout, one scale per 32 columns (Convert.swift:254-282). */
enum vp_format { VP_FMT_F16 = 0, VP_FMT_Q8 = 1, VP_FMT_Q4 = 2, VP_FMT_Q8G32 = 3 };

/* Matrix roles for vp_pack_matrix: the packer applies the row order the fused epilogues need. */
enum vp_matrix_kind {
  VP_MAT_PLAIN = 0,  /* O, down and the tied embedding / lm_head: natural row order */
  VP_MAT_QKV = 1,    /* [q(896); k(128); v(128)] rows of a layer: RoPE pairs (d, d+32) kept together */
  VP_MAT_GATEUP = 2  /* [gate(4864); up(4864)] rows: gate j and up j kept together */
};

enum vp_error {
  VP_OK = 0,
  VP_ERR_ARG = -1,     /* bad argument (null pointer, size out of range, unsupported format) */
  VP_ERR_CUDA = -2,    /* a CUDA runtime call failed; vp_last_error() has the text */
  VP_ERR_STATE = -3,   /* call out of order (e.g. verify before weights are set) */
  VP_ERR_NOMEM = -4,   /* device allocation failed */
  VP_ERR_DEVICE = -5   /* the device reported an error in vp_state.err */
};

/* Device-side error bits in vp_state.err. */
#define VP_DEV_ERR_TREE 1     /* malformed tree buffer */
#define VP_DEV_ERR_CTX 2      /* pos + rows would pass max_ctx */
#define VP_DEV_ERR_TIMEOUT 4  /* a bounded wait (mbarrier / copy) gave up */
#define VP_DEV_ERR_STEPS 8    /* out_tokens full */

typedef struct vp_ctx vp_ctx;

typedef struct {
  int32_t format;    /* enum vp_format */
  int32_t n_layers;  /* 1..24 (24 for Qwen2.5-0.5B) */
  int32_t vocab;     /* multiple of 16, e.g. 151936 */
  int32_t max_ctx;   /* KV slots per layer; must cover prefix + generated + VP_MAX_ROWS */
  int32_t max_steps; /* capacity of the committed-token buffer */
  int32_t device;    /* CUDA device ordinal */
} vp_config;

/* Device pass state (Shaders.swift:37-54 `State`, initialised by Engine.generate :945-964). */
typedef struct {
  int32_t pos;       /* KV slots holding committed context (first slot of the next pass) */
  int32_t n;         /* rows of the last pass */
  int32_t step;      /* committed tokens so far */
  int32_t done;      /* stop flag: set on EOS, max_steps or error; every kernel then returns */
  int32_t maxctx;
  int32_t maxsteps;
  int32_t eos0;
  int32_t eos1;
  int32_t nver;      /* rows whose argmax the next commit reads */
  int32_t vrow0;     /* first of those rows (n-1 after a prefill chunk, else 0) */
  int32_t passes;    /* committed passes (diagnostics, Shaders.swift:308) */
  int32_t accepted;  /* accepted drafts (diagnostics, Shaders.swift:324) */
  int32_t err;       /* VP_DEV_ERR_* bits */
  int32_t last_token;/* last committed token: row 0 of the next pass */
  int32_t mode;      /* 0 verify, 1 prefill (set by the pass's embed kernel) */
  int32_t advance;   /* prefill: rows to add to pos at commit */
} vp_state;

/* Borrowed, packed weights of one model (vp_pack_matrix output for matrices, fp32 vectors). */
typedef struct {
  const void* embed;                 /* [vocab][896], kind PLAIN; tied lm_head */
  const float* final_norm;           /* [896] */
  const void* wqkv[VP_MAX_LAYERS];   /* [1152][896], kind QKV */
  const float* bqkv[VP_MAX_LAYERS];  /* [1152] natural order q, k, v */
  const void* wo[VP_MAX_LAYERS];     /* [896][896] */
  const void* wgu[VP_MAX_LAYERS];    /* [9728][896], kind GATEUP */
  const void* wd[VP_MAX_LAYERS];     /* [896][4864] */
  const float* ln1[VP_MAX_LAYERS];   /* [896] input_layernorm */
  const float* ln2[VP_MAX_LAYERS];   /* [896] post_attention_layernorm */
} vp_weights;

/* ---- weight formats (replaces Convert.swift:254-370 output layouts + ModelFile.swift tensors) ----
 * Standard input layouts (what a converter writes):
 *   q4:  codes uint8 [rows][cols/2], weight 2j in the low nibble of byte j (Convert.swift:317);
 *        scales half2 [rows][cols/64] = (scale, min); w = scale*q + min (Convert.swift:290-317).
 *   q8:  codes int8 [rows][cols]; scales half [rows][cols/64]; w = scale*q (group 64).
 *   q8g32: codes int8 [rows][cols]; scales half [rows][cols/32]; w = scale*q (group 32, the
 *        reference's quantizeQ8 output, Convert.swift:254-282).
 *   f16: half [rows][cols]; scales NULL.
 * vp_pack_matrix rewrites one matrix into the kernel layout (16-row x 64-column tiles in
 * tensor-core fragment order). Both buffers are device memory. */
size_t vp_packed_bytes(int32_t format, int32_t rows, int32_t cols);
int vp_pack_matrix(int32_t format, int32_t kind, int32_t rows, int32_t cols, const void* d_codes,
                   const void* d_scales, void* d_out, void* stream);

/* ---- context (Engine.init, Engine.swift:71-232) ---- */
int vp_create(const vp_config* cfg, vp_ctx** out);
void vp_destroy(vp_ctx* ctx);
int vp_set_weights(vp_ctx* ctx, const vp_weights* w);
const char* vp_last_error(void);

/* ---- request set-up (Engine.generate state init, Engine.swift:937-964) ----
 * cached: KV slots already valid (shared prefix); max_new: tokens to generate (incl. a stop). */
int vp_begin(vp_ctx* ctx, int32_t cached, int32_t max_new, int32_t eos0, int32_t eos1, void* stream);

/* ---- prefix KV cache on disk (Engine.savePrefix / loadPrefix, Engine.swift:788-838) ----
 * Host copies of the K and V rows of the first n cached positions, laid out as the body of the
 * reference's prefix file: all K rows, then all V rows, each [layer][kv head][n][64] fp16.
 * vp_prefix_bytes gives the size (2 * layers * 2 * n * 128 bytes). vp_save_prefix copies device ->
 * host and synchronises `stream`; vp_load_prefix copies host -> device (stream-ordered), after
 * which vp_begin(ctx, n, ...) starts a request whose first n positions are that prefix. */
size_t vp_prefix_bytes(vp_ctx* ctx, int32_t n);
int vp_save_prefix(vp_ctx* ctx, int32_t n, void* host, void* stream);
int vp_load_prefix(vp_ctx* ctx, int32_t n, const void* host, void* stream);

/* ---- prefill (Engine.encodePrefill :588-601 = k_embed_prompt + 24 layers + lm_head + commit) ----
 * Runs n prompt tokens at slots pos..pos+n-1 in chunks of 16 rows, then the lm_head on the last
 * row and a 1-row greedy commit (k_commit, Shaders.swift:194-244): out_tokens[step] = argmax. */
int vp_prefill(vp_ctx* ctx, const int32_t* d_tokens, int32_t n, void* stream);

/* ---- verify pass (Engine.encodeWidePass :567-579 with the tree of k_ildraft) ----
 * tree: VP_TREE_INTS int32 (host or device pointer, copied with cudaMemcpyDefault). Runs embed,
 * 24 layers and lm_head with per-row argmax partials; does not commit. */
int vp_verify(vp_ctx* ctx, const int32_t* tree, void* stream);
/* Chain form: row 0 = last token, rows 1..nd = drafts (Shaders.swift:322 prefix acceptance). */
int vp_verify_chain(vp_ctx* ctx, const int32_t* drafts, int32_t nd, void* stream);

/* ---- accept / commit (k_commit_spec, Shaders.swift:254-365) ----
 * Argmax per row, longest matching tree path, committed tokens to out_tokens, pos += m+1,
 * KV compaction of the accepted rows. */
int vp_commit(vp_ctx* ctx, void* stream);

/* ---- whole pass: verify + commit as one persistent-kernel launch (the pass encoder) ---- */
int vp_pass(vp_ctx* ctx, const int32_t* tree, void* stream);
/* Passes of several requests in one launch (no counterpart in the reference, which serves one
 * request at a time, Engine.swift:567-579): up to 2 contexts (distinct, same device and format),
 * each with its tree (host or device pointer), run one verify pass + commit each, every request on
 * its own half of the SMs (its own barriers, state and scratch). A single pass is bound by the
 * latency of its dependent stages rather than by SMs or HBM, so two requests per launch nearly
 * double the committed tokens per second. Every request gets half the SMs also when n = 1: the
 * stage splits follow the CTA count, so a request stays bit-identical across its passes (tree ==
 * sequential) only if all of them run with the same share. Stream-ordered; contexts not used by
 * this call are untouched. */
int vp_pass_multi(vp_ctx* const* ctxs, const int32_t* const* trees, int32_t n, void* stream);
/* The same with an explicit share: every request runs on gridDim / shares CTAs (shares 1..4,
 * 1 <= n <= shares), with the same bit-identity rule: a request's passes must all run with one share.
 * vp_pass_multi(ctxs, trees, n, s) = vp_pass_batch(ctxs, trees, n, 2, s). With three or four shares
 * (37 to 49 CTAs per request on a B200) the QKV, O and down projections run one or two row-blocks per
 * CTA. Returns VP_ERR_ARG for a bad n / shares, VP_ERR_DEVICE if a share is below 36 SMs. */
int vp_pass_batch(vp_ctx* const* ctxs, const int32_t* const* trees, int32_t n, int32_t shares, void* stream);
/* Prefill of k requests (vp_prefill of each, Engine.encodePrefill :588-601) with every request on
 * gridDim / shares CTAs: launch c runs chunk c (16 rows) of every prompt that has one. A request
 * prefilled on a share and then decoded with vp_pass_batch on the same share gives the tokens of
 * its greedy 1-row passes on that share. d_tokens[i]: n[i] prompt ids on the device. */
int vp_prefill_batch(vp_ctx* const* ctxs, const int32_t* const* d_tokens, const int32_t* n, int32_t k,
                     int32_t shares, void* stream);

/* One step of the host's decode loop (the body of Engine.generate's loop, Engine.swift:937-1015:
 * fill State, encode the pass, wait, read State and the committed tokens) in one call from host
 * memory: optionally the 64-byte state (state_in, NULL to continue from the device state), the
 * tree (VP_TREE_INTS int32, host), one pass (verify + commit), then the state into state_out and,
 * if tokens_out is not NULL, the tokens this pass committed into tokens_out (VP_MAX_ROWS int32,
 * host: the committed tokens in order, then -1; all -1 when the request had already stopped).
 * Synchronises `stream`, also when it fails. The inputs go through the context's pinned staging
 * block in one host-to-device copy (state, token slots and tree are adjacent on the device), the
 * results in one device-to-host copy of 128 bytes; the copy in, the pass and the copy out are one
 * CUDA graph of the context (one per input form, captured on a stream of its own at the first call,
 * recaptured after vp_set_weights; three stream operations if a capture fails). Returns
 * VP_ERR_DEVICE when state_out->err is set. */
int vp_step(vp_ctx* ctx, const vp_state* state_in, const int32_t* tree, vp_state* state_out,
            int32_t* tokens_out, void* stream);

/* ---- results ---- */
int vp_read_state(vp_ctx* ctx, vp_state* host, void* stream);       /* syncs `stream` */
/* The host fills State (Engine.swift:937-964 writes the shared State buffer before a pass):
 * copies `state` (host memory, or device memory when from_device != 0) into the context's device
 * state, stream-ordered. Writing back a snapshot taken after a prefill replays later passes over
 * the same cached prefix: passes only write KV slots at or above the state's pos. */
int vp_write_state(vp_ctx* ctx, const vp_state* state, int32_t from_device, void* stream);
int vp_read_tokens(vp_ctx* ctx, int32_t* host, int32_t count, void* stream); /* syncs `stream` */
int32_t* vp_device_tokens(vp_ctx* ctx);   /* out_tokens, int32[max_steps], -1 = not yet written */
vp_state* vp_device_state(vp_ctx* ctx);

/* ---- parity helpers ----
 * Full fp32 logits [16][vocab] of the rows of the last verify pass or prefill chunk (the values
 * whose argmax the commit reduces). */
int vp_debug_logits(vp_ctx* ctx, float* d_out, void* stream);
/* Raw scratch buffers for tests: 0 x fp32[16][896], 1 q fp32[16][896], 2 KV cache K,
 * 3 KV cache V (half [layers][2][max_ctx][64]), 4 argmax partial values fp32 [16][parts],
 * 5 argmax partial ids int32 [16][parts] (parts = CTAs of the pass kernel), 6 stage trace of the
 * last launch: uint64 [256] %globaltimer ns (start, after embed, after each of the 5 stages of
 * every layer, after the lm_head, end), 7 the context's tree buffer (int32[VP_TREE_INTS]: a
 * drafter that writes it directly saves vp_pass its tree copy). */
int vp_buffer(vp_ctx* ctx, int32_t which, void** ptr, size_t* bytes);

/* ---- greedy lm-head argmax that allocates nothing ----
 * No counterpart in the reference (instantllm always owns its buffers); it exists for callers
 * that cannot allocate device memory: hosts whose device memory is entirely handed out by their
 * own pool or budget, and serving loops where a cudaMalloc / cudaFree would stall other work on
 * the device. tokens[r] = argmax_v of (RMSNorm(x[r]) * final_norm) . E[v] for r < rows (the tied
 * lm_head; lowest id on ties), the same arithmetic as the pass's own lm_head.
 *   format  VP_FMT_*; embed is the packed [vocab][896] matrix (vp_pack_matrix, VP_MAT_PLAIN)
 *   x       fp32 [rows][896] residual rows (device); tokens int32 [rows] (device)
 *   limits  1 <= rows <= VP_MAX_ROWS; vocab a multiple of 16, <= VP_NOALLOC_MAX_VOCAB;
 *           larger sizes return VP_ERR_ARG.
 * Scratch is one static device array inside the library (about 33 KiB, held by every GPU that
 * loads the library until the process exits). The first call on a device looks the array up on
 * that device (make that first call before any stream capture; a failed look-up is retried by the
 * next call). All calls share the array:
 * calls whose work overlaps on the GPU (other streams, other threads) race, so serialise them.
 * Runs on the current device and `stream`; reports a device-side timeout as token -1. */
#define VP_NOALLOC_MAX_VOCAB 163840
int vp_head_argmax_noalloc(int32_t format, int32_t vocab, const void* d_embed,
                           const float* d_final_norm, const float* d_x, int32_t rows,
                           int32_t* d_tokens, void* stream);

/* ---- two-stage lm-head over a 2-bit sketch (q4 only; probabilistic, off by default) ----
 * Replaces Engine.encodeSketchHead (Sources/Engine/Engine.swift:436-454) and the kernels
 * k_lmh_sketch_T / k_lmh_tau / k_lmh_exact_T (Shaders.swift:1377-1523). Stage 1 scores every
 * vocabulary row from the high two bits of its q4 codes with an uncertainty sigma for the dropped
 * low bits, and keeps per 32-row group the max of A - K sigma and A + K sigma; stage 2 recomputes
 * exact logits only in the groups whose upper bound reaches tau = max lower bound. The recomputed
 * logits are bit-identical to vp_head_argmax_noalloc's, so tokens[r] equals its token unless a
 * residual exceeds k_sigma sigma (the reference's default K is 6).
 *   hi       the reference's sketch plane (.ill tensor 291): uint8 [vocab][224], byte c holding
 *            codes 4c .. 4c+3 >> 2 (code 4c in bits 0-1); vp_pack_sketch packs it for the GPU
 *            into vp_sketch_bytes(vocab) bytes (device buffers, 16-byte aligned).
 *   embed    the packed q4 embedding (vp_pack_matrix, VP_FMT_Q4, VP_MAT_PLAIN)
 *   x        fp32 [rows][896] residual rows; tokens int32 [rows] (device)
 *   work     caller-owned device scratch of vp_sketch_work_bytes(vocab) bytes, 256-byte aligned:
 *            fp16 normed rows, RMSNorm partials, state, tau, the group bounds fp32 [2][16][ngrp]
 *            (ngrp = ceil(vocab / 32); lower bounds first) at offset vp_sketch_bounds_offset().
 *            Calls that share a work buffer must not overlap on the GPU.
 * Three launches: normed rows, stage 1 over every group, stage 2 over the candidates (its last CTA
 * writes tokens and ncand).
 *   ncand    optional int32[2] (device): groups that were candidates for row 0, for any row.
 *   limits   vocab a positive multiple of 16; 1 <= rows <= VP_MAX_ROWS; k_sigma > 0. */
size_t vp_sketch_bytes(int32_t vocab);
int vp_pack_sketch(int32_t vocab, const void* d_hi, void* d_out, void* stream);
size_t vp_sketch_work_bytes(int32_t vocab);
size_t vp_sketch_bounds_offset(void);
int vp_head_argmax_sketch(int32_t vocab, const void* d_embed, const void* d_sketch,
                          const float* d_final_norm, const float* d_x, int32_t rows, float k_sigma,
                          void* d_work, size_t work_bytes, int32_t* d_tokens, int32_t* d_ncand,
                          void* stream);

/* ---- the learned drafter on the device (k_ildraft, Shaders.swift:428-872; specification
 * tools/draft/ildraft.py:441-747; table loading ILDraft.swift:39-60) ----
 * vp_drafter_create parses an ILDRAFT1 table (the bytes of the file, host memory) and copies the
 * parts the drafter reads per step to `device`. vp_drafter_begin takes the request context the host
 * builds at request start (Drafter.begin, ildraft.py:452-516; ILDraft.swift:138): prompt ids, the
 * sorted distinct prompt ids (copy candidates), the nearest training documents (score, sequence =
 * the 5-token assistant tail + the document's output, and the sorted keys of the sequence's n-grams
 * of 1..MAXM tokens with the index after each one's first occurrence that has a next token), and
 * the association map (token -> max loglift, count; sorted by token) with the association
 * candidates. vp_draft runs one step on `stream`: from the request's output tokens (d_out_tokens:
 * d_state->step of them when d_state is given, which also makes a finished request (done) produce a
 * 1-row tree; else n_out) it grows the best-first tree of at most B (<= 15) drafts with `branch`
 * (<= 8) children per expansion and writes it to d_tree (VP_TREE_INTS int32, the verify pass's tree
 * buffer: row 0 the last output token). Passing a context's vp_device_tokens / vp_device_state and
 * then d_tree to vp_pass keeps the decode loop on the device. The optional debug block receives the
 * nodes (parents: -1 = root, -2 = unused; tokens), each expansion's top 8 (tokens -1 past the end,
 * probabilities float64) and a status (bit 0: more than 1024 candidates in a context, the rest
 * dropped). Errors: VP_ERR_ARG (bad table or sizes), VP_ERR_STATE (no request), VP_ERR_CUDA. */
#define VP_DRAFT_MAX_PROMPT 8192
typedef struct vp_drafter vp_drafter;
typedef struct {
  int32_t n_prompt; const int32_t* prompt;
  int32_t n_copy; const int32_t* copy;
  int32_t n_nb; const double* nb_score;
  const int32_t* nb_seq_off;   /* [n_nb + 1] */
  const int32_t* nb_seq;
  const int32_t* nb_key_off;   /* [n_nb + 1] */
  const uint64_t* nb_keys;     /* FNV-1a 64 of (order byte, tokens as u32 LE), ascending per document */
  const int32_t* nb_pos;
  int32_t n_as; const int32_t* as_tok; const double* as_max; const int32_t* as_cnt;
  int32_t n_as_cand; const int32_t* as_cand;
} vp_draft_request;
typedef struct {
  int32_t* parents;     /* device int32[15] */
  int32_t* tokens;      /* device int32[15] */
  int32_t* exp_tokens;  /* device int32[16][8] */
  double* exp_probs;    /* device double[16][8] */
  int32_t* status;      /* device int32[1] */
} vp_draft_debug;
int vp_drafter_create(const void* table, size_t bytes, int32_t device, vp_drafter** out);
void vp_drafter_destroy(vp_drafter* d);
int vp_drafter_begin(vp_drafter* d, const vp_draft_request* req);
int vp_draft(vp_drafter* d, const int32_t* d_out_tokens, const vp_state* d_state, int32_t n_out, int32_t B,
             int32_t branch, int32_t* d_tree, const vp_draft_debug* dbg, void* stream);

/* ---- CUDA graphs: the pass encoder as a replayable graph (the proposed vp_pass_graph) ----
 * vp_pass_graph captures one fused pass (vp_pass with the device tree d_tree; the context's own
 * tree buffer, vp_buffer 7, needs no copy node). vp_step_graph captures one step of the
 * device-resident decode loop: vp_draft from the context's device tokens and state into its tree
 * buffer, then vp_pass. vp_graph_launch replays a graph on a stream (stream-ordered, no
 * synchronisation). A graph holds the context's and the drafter request's device pointers by value:
 * a step graph refuses to launch once vp_drafter_begin has replaced its request (VP_ERR_STATE:
 * capture again), and graphs must be destroyed before their context or drafter. Errors: VP_ERR_ARG
 * (null argument, host tree), VP_ERR_STATE, VP_ERR_CUDA (capture or launch failed). */
typedef struct vp_graph vp_graph;
int vp_pass_graph(vp_ctx* ctx, const int32_t* d_tree, vp_graph** out);
int vp_step_graph(vp_ctx* ctx, vp_drafter* d, int32_t B, int32_t branch, vp_graph** out);
int vp_graph_launch(vp_graph* g, void* stream);
void vp_graph_destroy(vp_graph* g);

#ifdef __cplusplus
}
#endif
#endif /* VPASS_H */
