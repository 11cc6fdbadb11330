// Shared definitions of the verification-pass kernels (sm_100a).
//
// Layout vocabulary used throughout:
//  * tile: 16 weight rows x 64 columns (one quantisation group per row), stored in mma.sync
//    m16n8k16 A-fragment order so that each lane of a warp fetches its fragments with one
//    contiguous 16-byte (q4), 32-byte (q8) or 64-byte (f16) read. A matrix is [rows/16][cols/64]
//    tiles, row-block major.
//  * act block: 16 tokens x 64 columns of fp16 activations in m16n8k16 B-fragment order
//    (2 KiB; four 512-byte planes, one per 16-column k-step, lane L's 16 bytes at L*16).
//    Activations that feed a GEMM are produced directly in this order by the previous stage.
#pragma once
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/vpass.h"

namespace vp {

constexpr int H = VP_HIDDEN;
constexpr int F = VP_FFN;
constexpr int NQ = VP_NQ_HEADS;
constexpr int NKV = VP_NKV_HEADS;
constexpr int HD = VP_HEAD_DIM;
constexpr int QKV = VP_QKV_ROWS;
constexpr int ROWS = VP_MAX_ROWS;  // token rows per pass (MMA N dimension, always padded to 16)
constexpr int GS = VP_GROUP;
constexpr int HRB = H / 16;        // 56 row-blocks of a hidden-sized output
constexpr float EPS = 1e-6f;
constexpr float ATTN_SCALE = 0.125f;  // 64^-0.5, exact
constexpr int ATT_SUB = 32;           // virtual positions per attention record (fixed: shape-invariant)

// Bytes of one packed 16x64 tile per format: codes then per-row scale data (q8g32: two scales
// per row, one per 32-column half).
__host__ __device__ constexpr int tile_bytes(int fmt) {
  return fmt == VP_FMT_Q4 ? 512 + 64 : fmt == VP_FMT_Q8 ? 1024 + 32 : fmt == VP_FMT_Q8G32 ? 1024 + 64 : 2048;
}
__host__ __device__ constexpr int tile_code_bytes(int fmt) {
  return fmt == VP_FMT_Q4 ? 512 : (fmt == VP_FMT_Q8 || fmt == VP_FMT_Q8G32) ? 1024 : 2048;
}
__host__ __device__ constexpr bool fmt_is_q8(int fmt) { return fmt == VP_FMT_Q8 || fmt == VP_FMT_Q8G32; }
// Formats whose 64-column tile carries one scale per 32-column half: the group sums and the fold
// are kept per half.
__host__ __device__ constexpr bool fmt_halves(int fmt) { return fmt == VP_FMT_Q8G32; }
__host__ __device__ constexpr bool fmt_valid(int fmt) {
  return fmt == VP_FMT_F16 || fmt == VP_FMT_Q8 || fmt == VP_FMT_Q4 || fmt == VP_FMT_Q8G32;
}

// Half index of activation (token t, column k) in B-fragment order (see file comment).
__host__ __device__ inline int act_index(int t, int k) {
  const int G = k >> 6, kk = k & 63, j = kk >> 4, c = kk & 15;
  const int nt = t >> 3, gid = t & 7, tid4 = (c & 7) >> 1, reg = c >> 3, hi = c & 1;
  const int lane = gid * 4 + tid4, word = nt * 2 + reg;
  return G * 1024 + j * 256 + lane * 8 + word * 2 + hi;
}

// Per-pass row geometry, written by the pass's embed kernel and read by every later kernel.
struct RowInfo {
  int n;               // rows in this pass (1..16)
  int pos;             // slot of row 0
  int mode;            // 0 verify, 1 prefill chunk
  int live;            // 0: the request is done / errored, every kernel returns
  int depth[ROWS];
  int path[ROWS][ROWS];  // path[r][d]: row of r's ancestor at depth d (path[r][depth[r]] = r)
};

// Device scratch of one context (all pointers device memory).
struct Scratch {
  vp_state* st;
  RowInfo* ri;
  int32_t* tree;        // VP_TREE_INTS
  int32_t* out_tokens;  // max_steps
  int32_t* pass_tok;    // [16] tokens the last commit added to out_tokens, then -1
  float* x;             // [16][896] residual stream, fp32
  float* q;             // [16][896] roped queries, fp32
  __half* act_h;        // act blocks, K = 896: normed x for QKV / GU / lm_head
  __half* act_f;        // act blocks, K = 4864: SiLU(gate)*up for down
  float* ss;            // [HRB][16] per-row-block sums of squares of x (RMSNorm partials)
  uint64_t* act_ll;     // O output for gate/up: act blocks as (half2, flag) words [H * 16 / 2]
  uint64_t* ss_ll;      // its RMSNorm partials as (float, flag) words [HRB][16]
  uint64_t* q_ll;       // QKV output for the attention: roped queries as (float, flag) [16][896]
  uint64_t* kv_ll;      // and the pass rows' K / V as (half2, flag) words [K, V][kv head][16][32]
  uint64_t* att_ll;     // attention output for O: act blocks as (half2, flag) words [H * 16 / 2]
  uint64_t* dn_ll;      // down output for the next QKV: normed x as act blocks of (half2, flag) words
  uint64_t* dn_ss_ll;   // and its RMSNorm partials as (float, flag) words [HRB][16]
  uint64_t* dnp_ll;     // split down projection: the second CTA's partial tile of each row-block
                        // as (float, flag) words [HRB][128][2]
  uint32_t flag_q;      // flag of q_ll / kv_ll in this launch and layer
  float* part;          // split-K partial tiles [max units][16*16]
  int* tickets;         // split-K / attention arrival counters (self-resetting)
  float* att_part;      // attention split partials
  __half* kc;           // [layers][2][max_ctx][64]
  __half* vc;
  float2* rope;         // [max_ctx + 16][32] (cos, sin), angles computed in double
  float* pval;          // [16][vocab/16] per-row-block max logit
  int* pidx;            // [16][vocab/16] its id (lowest on ties)
  float* dbg_logits;    // [16][vocab] or null
  int max_ctx, max_steps, vocab, n_layers;
};

// ------------------------------------------------------------------------------------------
// PTX wrappers (sm_90+ bulk copies and mbarriers, sm_80+ mma.sync)

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// A thread whose phase is not complete is suspended (it issues nothing) until the phase completes
// or MBAR_SUSPEND_NS pass, so that waiting warps (the weight producer, consumers ahead of the ring)
// do not take issue slots from the warps of their SM sub-partition that compute.
constexpr uint32_t MBAR_SUSPEND_NS = 2000;
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(MBAR_SUSPEND_NS)
      : "memory");
  return ok != 0;
}

// Flagged words: 32 bits of data and a 32-bit flag written by one 8-byte store, so that a reader
// that sees the flag sees the data (no fence, no separate signal). Flags are unique per launch and
// layer; a reader polls until every word it needs carries the current flag.
__device__ __forceinline__ void st_flagged(uint64_t* p, uint32_t data, uint32_t flag) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((uint64_t)flag << 32) | data) : "memory");
}
__device__ __forceinline__ void ld_flagged2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

// Every device-side wait gives up after WAIT_NS of wall time (and after a poll cap), so a lost copy
// or a missing arrival can never hang the GPU: the caller records a timeout and returns.
constexpr unsigned long long WAIT_NS = 2000000000ull;  // 2 s

// Bounded wait on an mbarrier phase. Returns false on timeout.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity,
                                                  unsigned long long wait_ns = WAIT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 63 && globaltimer() - t0 > wait_ns) return false;
  }
  return false;
}

// Warp-uniform bounded wait: every lane probes the phase (each try_wait acquires for its own
// lane) and the warp leaves on a vote, so all 32 lanes leave together and the tensor-core
// instructions that follow (mma.sync.aligned) run converged. Returns the same value in every lane.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    if ((i & 63) == 63 && __any_sync(0xffffffffu, globaltimer() - t0 > WAIT_NS)) return false;
  }
  return false;
}

// One bulk copy global -> this CTA's shared memory, completing on `bar` (16-byte aligned, size a
// multiple of 16). Streaming weights are read once per pass: evict-first keeps them from pushing
// the activations and KV cache out of L2.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], "
      "%2, [%3], %4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// %globaltimer read issued only once `dep` is available (for timing a dependent chain).
__device__ __forceinline__ unsigned long long globaltimer_after(float dep) {
  unsigned long long t;
  asm volatile("{\n .reg .f32 z;\n add.f32 z, %1, 0f00000000;\n mov.u64 %0, %%globaltimer;\n}\n"
               : "=l"(t)
               : "f"(dep));
  return t;
}

// 16-byte cp.async global -> shared (bypasses L1); src_bytes 0 fills zeros. CTA barriers do not
// wait for these copies, so they can run ahead across barriers (unlike ordinary loads).
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes, uint64_t pol) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2, %3;" ::"r"(smem_u32(dst)),
               "l"(src), "r"(src_bytes), "l"(pol)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// D += A * B, m16n8k16, fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue (weight
// prefetch) now; wait until the previous kernel's memory is visible.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Barrier of the 512 compute threads of a CTA (named barrier 1). The persistent pass kernel adds a
// producer warp that never takes part in the compute stages, so stage code never uses
// __syncthreads.
constexpr int CONS_THREADS = 512;
// barrier.sync without .aligned: lanes of a warp may arrive from divergent code (a conditional
// store just before the barrier), which the .aligned form (bar.sync) leaves undefined; the
// __syncwarp reconverges the warp first.
__device__ __forceinline__ void cons_sync() {
  __syncwarp();
  asm volatile("barrier.sync 1, 512;" ::: "memory");
}
// Whole-CTA barrier after possibly divergent code (same reasoning as cons_sync).
__device__ __forceinline__ void cta_sync() {
  __syncwarp();
  __syncthreads();
}

__device__ __forceinline__ void set_error(vp_state* st, int bits) {
  atomicOr(&st->err, bits);
  atomicExch(&st->done, 1);
}

// RMSNorm scale 1 / sqrt(mean(x^2) + eps) of one token from its HRB per-row-block partial sums of
// squares, ld(r) giving partial r: four independent chains (partials r = c mod 4) added in a fixed
// order, a short dependent chain that every kernel normalising the same rows shares, so that all
// of them get the same bits.
template <typename Ld>
__device__ __forceinline__ float rms_inv(Ld ld) {
  float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int r = 0; r < HRB; ++r) a[r & 3] += ld(r);
  return 1.f / sqrtf(((a[0] + a[1]) + (a[2] + a[3])) / (float)H + EPS);
}

// Reduction helpers with a fixed combination order (results never depend on timing).
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace vp
