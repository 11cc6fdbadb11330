// Persistent verification-pass kernel: one launch runs embed, 24 layers, lm_head and the commit.
//
// Replaces the reference's per-dispatch pass encoder (Engine.encodeWidePass, Engine.swift:567-579:
// 171 Metal dispatches per pass) with one cooperative kernel, one CTA per SM:
//  * a stage hands its outputs to the next as flagged words (data and flag in one 8-byte store)
//    that the consumers poll; one grid barrier per layer (64-bit arrival counter, bounded spin)
//    remains, after gate/up;
//  * a producer warp streams the CTA's weights for the whole pass, in consumption order, as
//    contiguous pieces of up to 28 KiB (cp.async.bulk) into a 5-slot shared-memory ring with
//    full / empty mbarriers. Weights never depend on activations, so the stream runs up to the
//    ring's depth ahead, across stage boundaries, and overlaps the barrier and activation latency
//    of the dependent chain. Copies are few and large: each bulk-copy issue occupies the SM's copy
//    path for a few hundred cycles whatever its size;
//  * each CTA owns a contiguous row-block range of every GEMM stage it takes part in (the down
//    projection's row-blocks split in two K halves over two CTAs); a row-block's K groups are
//    split into a fixed number of parts that
//    different consumer warps process and that are summed in part order in shared memory;
//  * per-row arithmetic is a fixed function of the inputs (fixed parts, fixed group order, fixed
//    attention chunks), so tree rows reproduce 1-row passes bit for bit;
//  * the same pass body also runs as one of up to four requests in a launch (k_pass_groups), each
//    on its own share of the CTAs; the parts follow the share's CTA count, so a request reproduces
//    its 1-row passes bit for bit on the same share.
#pragma once
#include "vp_attn.cuh"
#include "vp_commit.cuh"
#include "vp_gemm.cuh"

namespace vp {

constexpr int MK_WARPS = 16;                     // consumer warps
constexpr int MK_CONS = MK_WARPS * 32;           // consumer threads (== PASS_THREADS)
constexpr int MK_THREADS = MK_CONS + 32;         // + the producer warp
constexpr int MK_NSLOT = 5;                      // weight ring slots
constexpr int MK_SLOT = 28672;                   // bytes per slot
constexpr int MK_PART_SLOTS = 24;                // partial tiles of a stage (1 KiB each)
// The RMSNorm partials of a normalising stage's input (HRB x 16 floats) are staged in the first
// MK_SS_SLOTS partial-tile slots and read while the jobs run, so those stages' jobs write their
// partial tiles past them.
constexpr int MK_SS_SLOTS = 4;
static_assert(MK_SS_SLOTS * 256 >= HRB * 16 && MK_SS_SLOTS + 16 <= MK_PART_SLOTS,
              "the staged RMSNorm partials and up to 16 jobs' partial tiles fit the partial area");
// Stage trace: trace[0, 256) holds CTA 0's %globaltimer after each grid barrier of a launch.
// Compiled with -DVP_TRACE_DETAIL (performance work only), every CTA also stamps the steps of
// layer MK_TRACE_LAYER (and of the lm_head stage) at trace[MK_TRACE_BASE + 256 * event + cta]:
// events 8 * stage + step for the GEMM stages (step 0 entry, 1 inputs in shared memory, 2 group
// sums, 3 jobs done, 4 pieces released, 5 epilogue done), 40 / 41 / 42 attention unit start /
// records done / combined, 48 + 2k / 49 + 2k arrival at / exit from the k-th grid barrier of the
// layer, 56 layer start, 64.. the attention units' steps, 192.. the down projection's tiles, and
// 288 + (warp * 5 + round) * 3 + s the lm_head jobs of each warp (s = 0 start, 1 first piece in
// the ring, 2 folded).
constexpr int MK_TRACE_BASE = 2048;
constexpr int MK_TRACE_LAYER = 5;
#ifdef VP_TRACE_DETAIL
constexpr int MK_TRACE = MK_TRACE_BASE + (64 + 16 * 8 + 96 + 16 * 5 * 3) * 256;
#define MK_CSTAMP(p, cond, ev)                                                                   \
  do {                                                                                           \
    if ((p).trace && threadIdx.x == 0 && (cond) && blockIdx.x < 256)                             \
      (p).trace[MK_TRACE_BASE + 256 * (ev) + blockIdx.x] = globaltimer();                        \
  } while (0)
#else
constexpr int MK_TRACE = MK_TRACE_BASE;
#define MK_CSTAMP(p, cond, ev) do {} while (0)
#endif
static_assert(MK_CONS == PASS_THREADS && MK_CONS == CONS_THREADS, "consumer warps run the stage code");

enum MkStage { MK_QKV = 0, MK_O = 1, MK_GU = 2, MK_DOWN = 3, MK_LM = 4 };
// Stage arrival counters of a launch (reset by the last CTA to exit): attention units and
// down-projection CTAs that have written their flagged outputs.
enum MkGate { MK_GATE_ATT = 0, MK_GATE_DOWN = 1, MK_GATES = 2 };
// Arrival count at which the consumers of a stage with `count` producers per layer start polling
// the flagged words of layer l: every producer of the layers before, which is always true by then,
// so the wait is one L2 round trip and a CTA barrier before the first poll. Measured on the
// config-2 pass (same box, interleaved runs): this 21.4 us per layer; waiting for 1/8, 1/4, 1/2 or
// all of layer l's producers 22.0, 22.1, 22.1 and 22.7; no counter at all 22.1; the producers'
// arrivals without the consumers' wait 21.9, the consumers' wait without arrivals 21.8. Both the
// producer's CTA barrier + add and the consumer's round trip + barrier before it polls help.
__device__ __forceinline__ unsigned mk_gate_target(int l, int count) {
  return (unsigned)(l * count);
}

// Parts per row-block (K split across the warps of one CTA) of a GEMM stage whose CTA owns nrb
// row-blocks, and K groups of each GEMM stage. Gate/up fills the 16 warps once: 4 row-blocks x 4
// parts or 5 x 3.
// SMALL: code for groups of fewer CTAs than a stage has row-blocks (three or four requests per
// launch, `k_pass_groups<FMT, true>`); the single-request kernel is compiled without it, so that
// its code stays as small as the one-row-block-per-CTA layout needs.
template <bool SMALL>
__host__ __device__ constexpr int mk_parts_g(int st, int nrb) {
  // QKV, O and down hold one row-block per CTA, or two in a small group: then half the parts each,
  // so the partial tiles still fit
  if constexpr (!SMALL) {
    return st == MK_QKV ? 14 : st == MK_O ? 14 : st == MK_DOWN ? 16
         : st == MK_GU ? (nrb >= 16 ? 1 : nrb <= 1 ? 14 : 16 / nrb) : 1;
  } else {
    return st == MK_QKV ? (nrb <= 1 ? 14 : 7) : st == MK_O ? (nrb <= 1 ? 14 : 7) : st == MK_DOWN ? (nrb <= 1 ? 16 : 8)
         : st == MK_GU ? (nrb >= 16 ? 1 : nrb <= 1 ? 14 : 16 / nrb) : 1;
  }
}
__host__ __device__ constexpr int mk_parts(int st, int nrb) { return mk_parts_g<true>(st, nrb); }
__host__ __device__ constexpr int mk_groups(int st) { return st == MK_DOWN ? F / GS : H / GS; }
__host__ __device__ constexpr int mk_chunk_groups(int fmt) {
  return fmt == VP_FMT_Q4 ? 7 : fmt == VP_FMT_Q8 ? 4 : 2;  // stand-alone k_gemm chunking
}
__host__ __device__ constexpr int mk_tiles_per_slot(int fmt) { return MK_SLOT / tile_bytes(fmt); }

// Contiguous row-block range [rb0, rb0 + n) of GEMM stage `st` owned by CTA `cta` of G. O and down
// go to CTAs 0..55 (which also keep their slice of x), QKV to the last 72 CTAs, gate/up and the
// lm_head in equal contiguous shares over every CTA. Weights stream ahead of the stages that use
// them, so the split balances each stage's work rather than each CTA's bytes. A group of fewer
// CTAs than a stage has row-blocks (36 to 71 CTAs: three or four requests per launch) takes QKV,
// O and down in equal contiguous shares too, one or two row-blocks per CTA.
__host__ __device__ constexpr bool mk_down_split(int G) { return G >= 2 * (H / 16); }
template <bool SMALL>
__host__ __device__ inline void mk_range_g(int st, int cta, int G, int nrb_lm, int& rb0, int& n) {
  rb0 = 0;
  n = 0;
  const int nh = H / 16, nq = QKV / 16, ngu = 2 * F / 16;
  if (st == MK_O || st == MK_DOWN) {
    if (SMALL && G < nh) { rb0 = cta * nh / G; n = (cta + 1) * nh / G - rb0; }
    else if (cta < nh) { rb0 = cta; n = 1; }
    else if (st == MK_DOWN && mk_down_split(G) && cta < 2 * nh) { rb0 = cta - nh; n = 1; }
  } else if (st == MK_QKV) {
    if (SMALL && G < nq) { rb0 = cta * nq / G; n = (cta + 1) * nq / G - rb0; }
    else if (cta >= G - nq) { rb0 = cta - (G - nq); n = 1; }
  } else if (st == MK_GU) {
    {
      rb0 = cta * ngu / G;  // < 2^31: 148 x 608
      n = (cta + 1) * ngu / G - rb0;
    }
  } else {
    rb0 = cta * nrb_lm / G;  // < 2^31 for every vocab the context accepts
    n = (cta + 1) * nrb_lm / G - rb0;
  }
}
__host__ __device__ inline void mk_range(int st, int cta, int G, int nrb_lm, int& rb0, int& n) {
  mk_range_g<true>(st, cta, G, nrb_lm, rb0, n);
}

// K-group window [g0, g0 + gn) of the row-blocks a CTA owns in stage st. The down projection is
// the longest stage (K = 4864: 76 tiles and 152 KB of activations per row-block); when the launch
// has 2 x 56 CTAs it runs on two CTAs per row-block: CTA r, which keeps row-block r's slice of x,
// takes groups 0..37, CTA 56 + r groups 38..75 and hands its partial tile to CTA r as flagged words
// (the first CTA adds it to its own: a fixed order).
__host__ __device__ inline void mk_window(int st, int cta, int G, int& g0, int& gn) {
  g0 = 0;
  gn = mk_groups(st);
  if (st == MK_DOWN && mk_down_split(G)) {
    const int half = (F / GS) / 2;
    if (cta < H / 16) {
      gn = half;
    } else {
      g0 = half;
      gn = F / GS - half;
    }
  }
}
__host__ __device__ inline int mk_pieces(int fmt, int nrb, int gn) {
  const int tiles = nrb * gn;
  const int tp = mk_tiles_per_slot(fmt);
  return (tiles + tp - 1) / tp;
}

struct MegaParams {
  Scratch s;
  const uint8_t* embed;
  const float* final_norm;
  const uint8_t* wqkv[VP_MAX_LAYERS];
  const float* bqkv[VP_MAX_LAYERS];
  const uint8_t* wo[VP_MAX_LAYERS];
  const uint8_t* wgu[VP_MAX_LAYERS];
  const uint8_t* wd[VP_MAX_LAYERS];
  const float* ln1[VP_MAX_LAYERS];
  const float* ln2[VP_MAX_LAYERS];
  int n_layers;
  int nrb_lm;                 // vocab / 16
  int max_chunks;             // attention records (32-position sub-chunks) per (row, kv head)
  unsigned long long* bar;    // grid barrier arrival counter (0 at launch, reset by the last CTA)
  unsigned* exit_ctr;         // CTAs that finished this launch
  unsigned* seq;              // launches so far: the flag of layer l is seq * 64 + l + 1
  unsigned* gate;             // [MK_GATES] stage arrival counters (0 at launch)
  unsigned long long* trace;  // CTA 0: %globaltimer after each stage (MK_TRACE entries)
  float* lm_pval;             // [16][gridDim] per-CTA argmax partials
  int* lm_pidx;
  // what this launch runs
  const int32_t* prompt;      // prefill chunk tokens (null: tree verify pass)
  int chunk_n, chunk_start, total_n;
  int do_lm, do_commit;
};

__device__ __forceinline__ const uint8_t* mk_weights(const MegaParams& p, int st, int l) {
  switch (st) {
    case MK_QKV: return p.wqkv[l];
    case MK_O: return p.wo[l];
    case MK_GU: return p.wgu[l];
    case MK_DOWN: return p.wd[l];
    default: return p.embed;
  }
}

// ---------------------------------------------------------------------------------------------
// grid barrier (consumer threads only)

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_add_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("red.release.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void mk_sync() { cons_sync(); }

// The CTA's writes before the barrier are ordered before its arrival by the CTA barrier + the release
// add (cumulativity); the acquire load orders the other CTAs' writes before what follows.
__device__ bool grid_barrier(const MegaParams& p, unsigned long long target, int* sAbort) {
  mk_sync();
  if (threadIdx.x == 0) {
    red_release_add_u64(p.bar, 1ull);
    bool ok = false;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 0; i < (1u << 26); ++i) {
      if (ld_acquire_u64(p.bar) >= target) { ok = true; break; }
      if ((i & 63) == 63 && globaltimer() - t0 > WAIT_NS) break;
      __nanosleep(32);
    }
    if (!ok) {
      set_error(p.s.st, VP_DEV_ERR_TIMEOUT);
      *sAbort = 1;
    }
  }
  mk_sync();
  return *(volatile int*)sAbort == 0;
}

// Gated flagged transport: a producer CTA writes its outputs as flagged words, then (after a CTA
// barrier) adds one to the stage's arrival counter with a relaxed atomic: no fence, since every
// word carries its own flag. A consumer CTA polls that one counter (one thread) until the target
// of mk_gate_target and only then polls the words themselves.
__device__ __forceinline__ void gate_arrive(unsigned* ctr) {
  asm volatile("red.relaxed.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}
__device__ __forceinline__ unsigned ld_relaxed_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// Bounded: a timeout sets the error bit and the CTA's abort flag. Ends with a CTA barrier.
__device__ void gate_wait(const unsigned* ctr, unsigned target, vp_state* st, volatile int* sAbort) {
  if (threadIdx.x == 0 && *sAbort == 0) {
    bool ok = false;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 0; i < (1u << 26); ++i) {
      if (ld_relaxed_u32(ctr) >= target) { ok = true; break; }
      if ((i & 63) == 63 && globaltimer() - t0 > WAIT_NS) break;
    }
    if (!ok) {
      set_error(st, VP_DEV_ERR_TIMEOUT);
      *sAbort = 1;
    }
  }
  mk_sync();
}

// ---------------------------------------------------------------------------------------------
// shared memory map

constexpr size_t MK_RING_BYTES = (size_t)MK_NSLOT * MK_SLOT;
constexpr size_t MK_ACT_BYTES = (size_t)(H / GS) * 2048;  // act blocks of a K = 896 GEMM
constexpr size_t MK_OFF_ACT = MK_RING_BYTES;
constexpr size_t MK_OFF_X = MK_OFF_ACT + MK_ACT_BYTES;            // group sums
constexpr size_t MK_X_BYTES = 2 * 16 * 16 * 4;  // group sums [14 groups][halves][16 tokens]
constexpr size_t MK_OFF_PART = MK_OFF_X + MK_X_BYTES;            // partial tiles
// The overlay holds, by stage: the act blocks, group sums and partial tiles of a GEMM stage; the
// attention scratch; the down projection's 16 partial tiles and 32 act staging buffers (15 below
// the partial tiles, 17 above).
constexpr size_t mk_max(size_t a, size_t b) { return a > b ? a : b; }
constexpr size_t MK_OVERLAY =
    mk_max(mk_max((sizeof(AttnSmem) + 127) & ~size_t(127), MK_ACT_BYTES + MK_X_BYTES + MK_PART_SLOTS * 1024),
           MK_ACT_BYTES + MK_X_BYTES + 16 * 1024 + 17 * 2048);
constexpr size_t MK_OFF_RS = MK_OFF_ACT + MK_OVERLAY;              // rscale[16]
constexpr size_t MK_OFF_LMV = MK_OFF_RS + 64;                     // [16 warps][16] best value
constexpr size_t MK_OFF_LMI = MK_OFF_LMV + 1024;                  // [16 warps][16] best id
constexpr size_t MK_OFF_RI = MK_OFF_LMI + 1024;                   // RowInfo copy
constexpr size_t MK_OFF_XRB = MK_OFF_RI + ((sizeof(RowInfo) + 15) & ~size_t(15));  // owned x slice
constexpr size_t MK_OFF_EPC = MK_OFF_XRB + 16 * 16 * 4;  // epilogue constants: 16 bias / norm weights,
                                                         // 128 (cos, sin) pairs
constexpr size_t MK_OFF_BAR = (MK_OFF_EPC + (16 + 256) * 4 + 127) & ~size_t(127);
constexpr size_t MK_OFF_GS = MK_OFF_BAR + 8 * (2 * MK_NSLOT);  // group sums ready (mbarrier)
constexpr size_t MK_SMEM = MK_OFF_GS + 8;
static_assert(sizeof(AttnSmem) <= MK_OFF_RS - MK_OFF_ACT, "attention scratch fits its overlay");
static_assert(MK_SMEM <= 232448, "dynamic shared memory of the pass kernel fits one sm_100 CTA");

// Consumer view of the weight ring: pieces are numbered over the whole pass in consumption order.
struct MkRing {
  uint8_t* base;
  uint64_t* full;   // [MK_NSLOT], producer arrive + transaction bytes
  uint64_t* empty;  // [MK_NSLOT], one arrival per consumer warp
  int released;     // pieces this warp has released (identical in all lanes)
  int waited;       // pieces this warp has seen full
  uint64_t* gsum;   // mbarrier: the H / GS group-sum warps of a stage wrote their sums
  uint32_t gs_phase;  // phases of gsum completed so far (its parity is the next wait's)
};

// ---------------------------------------------------------------------------------------------
// producer warp: issues every piece of the pass in order (lane 0)

template <int FMT, bool SMALL>
__device__ void mk_producer(const MegaParams& p, uint8_t* smem, volatile int* sStop, int cta, int G) {
  if ((threadIdx.x & 31) != 0) return;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + MK_OFF_BAR);
  uint64_t* empty = full + MK_NSLOT;
  constexpr int TB = tile_bytes(FMT);
  const int tp = mk_tiles_per_slot(FMT);
  const uint64_t pol = policy_evict_first();
  int k = 0;  // pieces issued
  bool ok = true;
  const int nst = p.n_layers * 4 + (p.do_lm ? 1 : 0);
  for (int si = 0; si < nst && ok; ++si) {
    const int l = si / 4, st = si < p.n_layers * 4 ? si % 4 : MK_LM;
    int rb0, nrb, g0, gn;
    mk_range_g<SMALL>(st, cta, G, p.nrb_lm, rb0, nrb);
    if (nrb == 0) continue;
    mk_window(st, cta, G, g0, gn);
    const int ng = mk_groups(st);
    const int tiles = nrb * gn;  // a window narrower than the row-block only when nrb == 1
    const uint8_t* src = mk_weights(p, st, l) + ((size_t)rb0 * ng + g0) * TB;
    for (int t0 = 0; t0 < tiles && ok; t0 += tp, ++k) {
      const int slot = k % MK_NSLOT;
      if (k >= MK_NSLOT) {
        // the slot's previous piece must be released by every consumer warp
        const uint32_t par = ((k / MK_NSLOT) - 1) & 1;
        bool got = false;
        const unsigned long long t0 = globaltimer();
        for (uint32_t i = 0; i < (1u << 26); ++i) {
          if (mbar_try_wait(empty + slot, par)) { got = true; break; }
          if (*sStop || ((i & 15) == 15 && globaltimer() - t0 > WAIT_NS)) break;
        }
        if (!got) { ok = false; break; }
      }
      const uint32_t bytes = (uint32_t)(min(tp, tiles - t0) * TB);
      mbar_arrive_expect_tx(full + slot, bytes);
      bulk_g2s(smem + (size_t)slot * MK_SLOT, src + (size_t)t0 * TB, bytes, full + slot, pol);
    }
  }
  // every issued piece lands before the CTA's shared memory is released: only the last piece of
  // each slot can still be in flight
  for (int s = 0; s < MK_NSLOT; ++s) {
    int last = -1;
    for (int q = s; q < k; q += MK_NSLOT) last = q;
    if (last >= 0) mbar_wait_bounded(full + s, (last / MK_NSLOT) & 1);
  }
}

// ---------------------------------------------------------------------------------------------
// consumer GEMM stage

__device__ __forceinline__ uint4 act_frag_smem(const uint8_t* sAct, int g, int j, int lane) {
  return *reinterpret_cast<const uint4*>(sAct + (size_t)g * 2048 + j * 512 + lane * 16);
}

// acc += NT consecutive tiles (groups g .. g+NT-1 of the row-block) times their activations. The
// tiles' MMA chains are independent (instruction-level parallelism); their folds into acc run in
// group order, so the result equals NT single-tile steps.
// GLOBAL_B: the activations come from global memory (down projection: K = 4864 does not fit in
// shared memory) and the group sums are formed from the fragments; otherwise both are in smem.
template <int FMT, bool GLOBAL_B, int NT>
__device__ __forceinline__ void mk_tiles_bf(const uint8_t* const (&tile)[NT], int g, const uint4 (&bf)[NT][4],
                                            const float* sX, int lane, float (&acc)[2][4]) {
  const int gid = lane >> 2, tid4 = lane & 3;
  if constexpr (FMT == VP_FMT_F16) {
#pragma unroll
    for (int u = 0; u < NT; ++u) {
      uint32_t w[4][4];
      load_a_frags_all<FMT>(tile[u], lane, w);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        mma16816(acc[0], w[j][0], w[j][1], w[j][2], w[j][3], bf[u][j].x, bf[u][j].y);
        mma16816(acc[1], w[j][0], w[j][1], w[j][2], w[j][3], bf[u][j].z, bf[u][j].w);
      }
    }
  } else {
    // NH = 2 for q8g32: the two 32-column halves of a tile accumulate, sum and fold separately
    constexpr int NH = fmt_halves(FMT) ? 2 : 1;
    float ag[NT][NH][2][4];
    float tx[NT][NH][2][2];
#pragma unroll
    for (int u = 0; u < NT; ++u) {
#pragma unroll
      for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) ag[u][h][nt][i] = 0.f;
      if constexpr (GLOBAL_B) {
        // group sums from the fragments just loaded: a ones-matrix MMA
        const uint32_t ONE2 = 0x3C003C00u;
        float xs[NH][2][4] = {};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int h = NH == 2 ? (j >> 1) : 0;
          mma16816(xs[h][0], ONE2, ONE2, ONE2, ONE2, bf[u][j].x, bf[u][j].y);
          mma16816(xs[h][1], ONE2, ONE2, ONE2, ONE2, bf[u][j].z, bf[u][j].w);
        }
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          tx[u][h][0][0] = xs[h][0][0]; tx[u][h][0][1] = xs[h][0][1];
          tx[u][h][1][0] = xs[h][1][0]; tx[u][h][1][1] = xs[h][1][1];
        }
      } else {
#pragma unroll
        for (int h = 0; h < NH; ++h) {
          const float* xg = sX + ((g + u) * NH + h) * 16;
          const float2 x0 = *reinterpret_cast<const float2*>(xg + 2 * tid4);
          const float2 x1 = *reinterpret_cast<const float2*>(xg + 8 + 2 * tid4);
          tx[u][h][0][0] = x0.x; tx[u][h][0][1] = x0.y; tx[u][h][1][0] = x1.x; tx[u][h][1][1] = x1.y;
        }
      }
    }
    uint32_t w[NT][4][4];
#pragma unroll
    for (int u = 0; u < NT; ++u) load_a_frags_all<FMT>(tile[u], lane, w[u]);
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int u = 0; u < NT; ++u) {
        const int h = NH == 2 ? (j >> 1) : 0;
        mma16816(ag[u][h][0], w[u][j][0], w[u][j][1], w[u][j][2], w[u][j][3], bf[u][j].x, bf[u][j].y);
        mma16816(ag[u][h][1], w[u][j][0], w[u][j][1], w[u][j][2], w[u][j][3], bf[u][j].z, bf[u][j].w);
      }
#pragma unroll
    for (int u = 0; u < NT; ++u) {
      float sf[NH][2], sb[NH][2];
      if constexpr (NH == 2) load_fold_halves(tile[u], gid, sf, sb);
      else load_fold<FMT>(tile[u], gid, sf[0], sb[0]);
#pragma unroll
      for (int h = 0; h < NH; ++h)
#pragma unroll
        for (int nt = 0; nt < 2; ++nt)
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int r = i >> 1;
            acc[nt][i] = fmaf(sf[h][r], ag[u][h][nt][i], fmaf(sb[h][r], tx[u][h][nt][i & 1], acc[nt][i]));
          }
    }
  }
}

template <int FMT, int NT>
__device__ __forceinline__ void mk_tiles(const uint8_t* const (&tile)[NT], int g, const uint8_t* sAct,
                                         const float* sX, int lane, float (&acc)[2][4]) {
  uint4 bf[NT][4];
#pragma unroll
  for (int u = 0; u < NT; ++u)
#pragma unroll
    for (int j = 0; j < 4; ++j) bf[u][j] = act_frag_smem(sAct, g + u, j, lane);
  mk_tiles_bf<FMT, false, NT>(tile, g, bf, sX, lane, acc);
}
// Down projection: two 2 KiB staging buffers of act blocks per warp, so that two blocks are in
// flight while a third computes. In that stage the overlay holds only the 16 partial tiles (at
// MK_OFF_PART); the 32 buffers fill the rest of it: 15 below the partial tiles (the act blocks and
// group sums areas), 17 above them.
constexpr int MK_DOWN_BUFS = 2 * MK_WARPS;
constexpr size_t MK_DOWN_LOW = (MK_OFF_PART - MK_OFF_ACT) / 2048;                    // 15
constexpr size_t MK_DOWN_HIGH = MK_OFF_PART - MK_OFF_ACT + (size_t)mk_parts(MK_DOWN, 1) * 1024;
static_assert(MK_DOWN_LOW == 15, "act blocks + group sums hold 15 staging buffers");
static_assert(MK_DOWN_HIGH + (MK_DOWN_BUFS - MK_DOWN_LOW) * 2048 <= MK_OVERLAY,
              "down-projection staging buffers fit the overlay past the partial tiles");
__device__ __forceinline__ uint8_t* mk_down_stage(uint8_t* smem, int b) {
  return smem + MK_OFF_ACT + (b < (int)MK_DOWN_LOW ? (size_t)b * 2048 : MK_DOWN_HIGH + (size_t)(b - MK_DOWN_LOW) * 2048);
}

// Wait until piece k is in the ring (bounded); returns its slot base or null on timeout.
__device__ __forceinline__ const uint8_t* mk_piece(MkRing& rg, int k) {
  while (rg.waited <= k) {
    if (!mbar_wait_warp(rg.full + rg.waited % MK_NSLOT, (rg.waited / MK_NSLOT) & 1)) return nullptr;
    ++rg.waited;
  }
  return rg.base + (size_t)(k % MK_NSLOT) * MK_SLOT;
}
// Release every piece below k (this warp is done with them). A piece is released only after it
// has landed: the slot's empty barrier then counts exactly one arrival per warp per piece, because
// the producer issues piece r + MK_NSLOT only after every warp released piece r. Returns false on
// timeout.
// Pieces are released one at a time, each as soon as it has landed, so a warp never waits for a
// piece while it still holds an older one (the newer piece may need the older one's slot).
__device__ __forceinline__ bool mk_release(MkRing& rg, int k, int lane) {
  for (; rg.released < k; ++rg.released) {
    if (!mk_piece(rg, rg.released)) return false;
    __syncwarp();
    if (lane == 0)
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(rg.empty + rg.released % MK_NSLOT))
                   : "memory");
  }
  return true;
}

// The job loop of a GEMM stage for one warp. Writes the partial tile of each job to the
// partial-tile area, or (lm_head, one part) folds it into this warp's running argmax in shared
// memory.
struct MkJobs {
  int piece0, rb0, nrb, P, ng;
  float* part;           // partial tile of job j at part + j * 256
  uint64_t* gsum;        // non-null: wait for this phase of the group-sum mbarrier before the
  uint32_t gs_parity;    // first tile (the fold reads the group sums)
  const __half* actg;    // down projection: act blocks of the SiLU output
  unsigned long long* trace;  // performance tracing only (null: off)
};
// What a stage's jobs are, fixed at compile time so that each stage's code holds only its own
// loop (instruction-cache footprint): activations in shared memory and partial tiles out (QKV,
// O, gate/up), activations streamed from global memory (down), or a running argmax (lm_head).
enum MkJobKind { JOB_SMEM = 0, JOB_DOWN = 1, JOB_ARGMAX = 2 };

// The ring state travels by value (registers) and comes back updated: x = pieces released (or -1
// after a timeout), y = pieces seen full.
template <int FMT, int KIND>
__device__ __forceinline__ int2 mk_jobs(const MkJobs J, MkRing rg, uint8_t* smem) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tid4 = lane & 3;
  uint8_t* sAct = smem + MK_OFF_ACT;
  float* sX = reinterpret_cast<float*>(smem + MK_OFF_X);
  float* sPart = J.part;
  const float* sRs = reinterpret_cast<const float*>(smem + MK_OFF_RS);
  float* sLmV = reinterpret_cast<float*>(smem + MK_OFF_LMV);
  int* sLmI = reinterpret_cast<int*>(smem + MK_OFF_LMI);
  const int piece0 = J.piece0, rb0 = J.rb0, nrb = J.nrb, P = J.P, ng = J.ng;
  constexpr bool down = KIND == JOB_DOWN;
  const int tp = mk_tiles_per_slot(FMT);
  constexpr int TB = tile_bytes(FMT);
  // jobs (row-block i, part q) -> warp (i * P + q) % 16, in increasing tile order per warp
  const int jobs = nrb * P;
  bool ok = true;
  if (J.gsum && warp < jobs) ok = mbar_wait_warp(J.gsum, J.gs_parity);
  for (int j = warp; j < jobs && ok; j += MK_WARPS) {
    const int i = j / P, q = j % P;
    const int ga = q * ng / P, gb = (q + 1) * ng / P;
    float acc[2][4] = {};
#ifdef VP_TRACE_DETAIL
    unsigned long long* ltr = (KIND == JOB_ARGMAX && J.trace && j / MK_WARPS < 5 && lane == 0)
                                  ? J.trace + MK_TRACE_BASE + (size_t)(288 + (warp * 5 + j / MK_WARPS) * 3) * 256 + blockIdx.x
                                  : nullptr;
    if (ltr) ltr[0] = globaltimer();
#endif
    if constexpr (down) {
      // one tile per step, software-pipelined: the act blocks of tiles g + 1 and g + 2 stream from
      // L2 into this warp's two staging buffers (cp.async, each lane its own fragments) while tile
      // g computes from registers; the first copies overlap the wait for the weights
      uint8_t* const sB[2] = {mk_down_stage(smem, 2 * warp), mk_down_stage(smem, 2 * warp + 1)};
      const uint64_t pol = policy_evict_last();
      auto fetch = [&](int g) {
        uint8_t* b = sB[(g - ga) & 1];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          cp_async16(b + j * 512 + lane * 16, J.actg + (size_t)g * 1024 + j * 256 + lane * 8, 16u, pol);
        cp_async_commit();
      };
      if (ga < gb) fetch(ga);
      if (ga + 1 < gb) fetch(ga + 1);
#ifdef VP_TRACE_DETAIL
      // per-tile stamps of warps 0..3 of the traced layer: [warp][tile][piece ready, act landed, done]
      unsigned long long* dtr = (J.trace && warp < 4) ? J.trace + MK_TRACE_BASE + 192 * 256 + blockIdx.x : nullptr;
      auto dst = [&](int k, float dep) {
        if (dtr) { const unsigned long long v = globaltimer_after(dep); if (lane == 0) dtr[256 * k] = v; }
      };
#endif
      for (int g = ga; g < gb; ++g) {
        const int idx = i * ng + g;
        const int k = piece0 + idx / tp;
        if (!mk_release(rg, k, lane)) { ok = false; break; }
        const uint8_t* base = mk_piece(rg, k);
        if (!base) { ok = false; break; }
#ifdef VP_TRACE_DETAIL
        dst(warp * 24 + (g - ga) * 3 + 0, __uint_as_float(*reinterpret_cast<const uint32_t*>(base)));
#endif
        if (g + 1 < gb) cp_async_wait<1>();  // block g landed (g + 1 may still be in flight)
        else cp_async_wait<0>();
        __syncwarp();  // converged before the warp-collective MMAs
        uint4 bf[1][4];
        const uint8_t* b = sB[(g - ga) & 1];
#pragma unroll
        for (int j = 0; j < 4; ++j) bf[0][j] = *reinterpret_cast<const uint4*>(b + j * 512 + lane * 16);
#ifdef VP_TRACE_DETAIL
        dst(warp * 24 + (g - ga) * 3 + 1, __uint_as_float(bf[0][3].w));
#endif
        __syncwarp();  // every lane holds its fragments before the buffer is refilled
        if (g + 2 < gb) fetch(g + 2);
        const uint8_t* const tt[1] = {base + (size_t)(idx % tp) * TB};
        mk_tiles_bf<FMT, true, 1>(tt, g, bf, sX, lane, acc);
#ifdef VP_TRACE_DETAIL
        dst(warp * 24 + (g - ga) * 3 + 2, acc[1][3]);
#endif
      }
      cp_async_wait<0>();
    } else {
      for (int g = ga; g < gb; g += 2) {
        // tiles g and g+1 (if in the part): release the pieces before g's, wait for both
        const int idx = i * ng + g;
        const int k = piece0 + idx / tp;
        if (!mk_release(rg, k, lane)) { ok = false; break; }
        const uint8_t* base = mk_piece(rg, k);
        if (!base) { ok = false; break; }
#ifdef VP_TRACE_DETAIL
        if (ltr && g == ga) ltr[256] = globaltimer();
#endif
        const uint8_t* t0 = base + (size_t)(idx % tp) * TB;
        if (g + 1 < gb) {
          const int k1 = piece0 + (idx + 1) / tp;
          const uint8_t* base1 = mk_piece(rg, k1);
          if (!base1) { ok = false; break; }
          const uint8_t* const tt[2] = {t0, base1 + (size_t)((idx + 1) % tp) * TB};
          mk_tiles<FMT, 2>(tt, g, sAct, sX, lane, acc);
        } else {
          const uint8_t* const tt[1] = {t0};
          mk_tiles<FMT, 1>(tt, g, sAct, sX, lane, acc);
        }
      }
    }
    if (!ok) break;
    if constexpr (KIND == JOB_ARGMAX) {
      // lm_head: running best (value, lowest id) per token over this warp's row-blocks
      const int rb = rb0 + i;
      const int v0 = rb * 16 + gid, v1 = v0 + 8;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int t = nt * 8 + 2 * tid4 + e;
          const float l0 = acc[nt][e] * sRs[t], l1 = acc[nt][2 + e] * sRs[t];
          float bv = l0;
          int bi = v0;
          if (l1 > bv) { bv = l1; bi = v1; }
#pragma unroll
          for (int o = 4; o < 32; o <<= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
          }
          if (gid == 0) {  // this warp's running best of token t (shared memory, warp-private)
            float& mv = sLmV[warp * 16 + t];
            int& mi = sLmI[warp * 16 + t];
            if (bv > mv || (bv == mv && bi < mi)) { mv = bv; mi = bi; }
          }
        }
#ifdef VP_TRACE_DETAIL
      if (ltr) ltr[512] = globaltimer_after(sLmV[warp * 16]);
#endif
    } else {
      float* part = sPart + j * 256;
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int r = 0; r < 4; ++r)
          // [row half][token][row & 7]: the epilogue's lanes (8 rows of a token, 4 tokens per
          // warp) then read 32 consecutive words, free of bank conflicts
          part[(r >> 1) * 128 + (nt * 8 + 2 * tid4 + (r & 1)) * 8 + gid] = acc[nt][r];
    }
  }
  return make_int2(ok ? rg.released : -1, rg.waited);
}

// Fused epilogue of a GEMM stage, element-parallel over the CTA's 512 compute threads: thread
// (row-block i, token t, row pair rp) sums the K parts of output rows rp and rp + 8 (the RoPE pair
// of QKV, gate and up of gate/up, two dims of O / down) in part order and applies the stage's
// epilogue. The 8 lanes of a token sit in one warp (RMSNorm partial of the down / O output).
template <int MODE, bool SMALL>
__device__ __forceinline__ void mk_epilogue(const GemmParams& gp, int rb0, int nrb, int P, const float* sPart,
                                            const float* rs, const float* sEpc) {
  const Scratch& s = gp.s;
  const RowInfo* ri = s.ri;
  const int n = ri->n;
  if constexpr (MODE == MODE_SILU) {
    // up to 5 row-blocks (640 elements) on 512 threads: a thread's two elements are summed
    // together, so that the second one does not wait for the first one's latency chain
    const int ne = nrb * 128;
    for (int e0 = threadIdx.x; e0 < ne; e0 += 2 * MK_CONS) {
      const bool two = e0 + MK_CONS < ne;
      const int e[2] = {e0, two ? e0 + MK_CONS : e0};
      float g[2] = {0.f, 0.f}, u[2] = {0.f, 0.f};
      for (int q = 0; q < P; ++q)
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const float* part = sPart + (e[k] >> 7) * P * 256 + q * 256 + ((e[k] & 127) >> 3) * 8 + (e[k] & 7);
          g[k] += part[0];
          u[k] += part[128];
        }
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        const int lt = e[k] & 127, t = lt >> 3, f = (rb0 + (e[k] >> 7)) * 8 + (lt & 7);
        float h = 0.f;
        if (t < n) {
          const float gg = g[k] * rs[t];
          const float uu = u[k] * rs[t];
          h = gg / (1.f + expf(-gg)) * uu;
        }
        if (k == 0 || two) gp.act_out[act_index(t, f)] = __float2half_rn(h);
      }
    }
    return;
  } else {  // QKV, O, down: one 16-row block (128 elements) per CTA
  for (int e = threadIdx.x; e < nrb * 128; e += MK_CONS) {
    const int i = e >> 7, lt = e & 127, t = lt >> 3, rp = lt & 7, rb = rb0 + i;
    float s0 = 0.f, s1 = 0.f;
    const float* part = sPart + i * P * 256;
    for (int q = 0; q < P; ++q) {
      s0 += part[q * 256 + t * 8 + rp];
      s1 += part[q * 256 + 128 + t * 8 + rp];
    }
    if constexpr (MODE == MODE_RESID) {
      if (gp.part_ll_out) {  // second CTA of a split down projection: its partial goes to the first
        st_flagged(gp.part_ll_out + (size_t)rb * 256 + lt * 2, __float_as_uint(s0), gp.flag);
        st_flagged(gp.part_ll_out + (size_t)rb * 256 + lt * 2 + 1, __float_as_uint(s1), gp.flag);
        continue;  // uniform over the CTA
      }
      if (gp.part_ll_in) {  // first CTA: add the second CTA's partial (bounded poll)
        const uint64_t* w = gp.part_ll_in + (size_t)rb * 256 + lt * 2;
        uint64_t a = 0, b = 0;
        bool got = false;
        const unsigned long long t0 = globaltimer();
        for (uint32_t it = 0; it < (1u << 26); ++it) {
          ld_flagged2(w, a, b);
          if ((uint32_t)(a >> 32) == gp.flag && (uint32_t)(b >> 32) == gp.flag) { got = true; break; }
          if ((it & 15) == 15 && globaltimer() - t0 > WAIT_NS) break;
        }
        if (!got) set_error(s.st, VP_DEV_ERR_TIMEOUT);
        s0 = s0 + (got ? __uint_as_float((uint32_t)a) : 0.f);
        s1 = s1 + (got ? __uint_as_float((uint32_t)b) : 0.f);
      }
    }
    if constexpr (MODE == MODE_QKV) {
      const int head = rb >> 2, d = (rb & 3) * 8 + rp;
      float a = 0.f, b = 0.f;
      if (t < n) {
        // bias and rotations of the CTA's first row-block are in shared memory; a second one
        // (groups of fewer than 72 CTAs) reads them from global memory
        const bool first = !SMALL || i == 0;
        a = s0 * rs[t] + (first ? sEpc[rp] : gp.bias[head * HD + d]);
        b = s1 * rs[t] + (first ? sEpc[8 + rp] : gp.bias[head * HD + d + 32]);
        if (head < NQ + NKV) {
          const float2 cs = first ? reinterpret_cast<const float2*>(sEpc + 16)[lt]
                                  : s.rope[(ri->pos + ri->depth[t]) * 32 + d];
          const float a2 = a * cs.x - b * cs.y;
          const float b2 = b * cs.x + a * cs.y;
          a = a2; b = b2;
        }
      }
      // the attention polls flagged copies (no grid barrier between QKV and attention); the
      // plain q and the KV cache stay the record that later passes and the debug buffers read
      if (head < NQ) {  // uniform over each warp (4 warps per row-block)
        if (t < n) {
          s.q[t * H + head * HD + d] = a;
          s.q[t * H + head * HD + d + 32] = b;
          st_flagged(s.q_ll + t * H + head * HD + d, __float_as_uint(a), s.flag_q);
          st_flagged(s.q_ll + t * H + head * HD + d + 32, __float_as_uint(b), s.flag_q);
        }
      } else {
        const int kind = head < NQ + NKV ? 0 : 1, kvh = kind == 0 ? head - NQ : head - NQ - NKV;
        const __half ha = __float2half_rn(a), hb = __float2half_rn(b);
        if (t < n) {
          __half* row = (kind == 0 ? s.kc : s.vc) + ((size_t)(gp.layer * NKV + kvh) * s.max_ctx + ri->pos + t) * HD;
          row[d] = ha;
          row[d + 32] = hb;
        }
        // dims (d, d + 1) are one flagged word: the even lane takes its neighbour's half
        const uint32_t ua = __half_as_ushort(ha), ub = __half_as_ushort(hb);
        const uint32_t na = __shfl_down_sync(0xffffffffu, ua, 1), nb = __shfl_down_sync(0xffffffffu, ub, 1);
        if (t < n && (rp & 1) == 0) {
          uint64_t* w = s.kv_ll + ((size_t)(kind * NKV + kvh) * ROWS + t) * (HD / 2);
          st_flagged(w + d / 2, ua | (na << 16), s.flag_q);
          st_flagged(w + (d + 32) / 2, ub | (nb << 16), s.flag_q);
        }
      }
    } else if constexpr (MODE == MODE_RESID) {
      const int d0 = rb * 16 + rp, d1 = d0 + 8;
      float v0 = 0.f, v1 = 0.f;
      if (t < n) {
        const float x0 = gp.xs ? gp.xs[t * 16 + rp] : __ldcg(s.x + t * H + d0);
        const float x1 = gp.xs ? gp.xs[t * 16 + rp + 8] : __ldcg(s.x + t * H + d1);
        v0 = x0 + s0;
        v1 = x1 + s1;
        if (gp.xs) {
          gp.xs[t * 16 + rp] = v0;
          gp.xs[t * 16 + rp + 8] = v1;
        }
        s.x[t * H + d0] = v0;
        s.x[t * H + d1] = v1;
      }
      const float w0 = nrb == 1 ? sEpc[rp] : gp.wnext[d0], w1 = nrb == 1 ? sEpc[rp + 8] : gp.wnext[d1];
      const __half h0 = __float2half_rn(v0 * w0), h1 = __float2half_rn(v1 * w1);
      float sq = v0 * v0 + v1 * v1;
      sq += __shfl_xor_sync(0xffffffffu, sq, 1);
      sq += __shfl_xor_sync(0xffffffffu, sq, 2);
      sq += __shfl_xor_sync(0xffffffffu, sq, 4);
      if (gp.act_ll_out) {
        // columns (d, d + 1) of token t are one flagged word: the even lane takes its neighbour's
        const uint32_t b0 = __half_as_ushort(h0), b1 = __half_as_ushort(h1);
        const uint32_t n0 = __shfl_down_sync(0xffffffffu, b0, 1), n1 = __shfl_down_sync(0xffffffffu, b1, 1);
        if ((rp & 1) == 0) {
          st_flagged(gp.act_ll_out + act_index(t, d0) / 2, b0 | (n0 << 16), gp.flag);
          st_flagged(gp.act_ll_out + act_index(t, d1) / 2, b1 | (n1 << 16), gp.flag);
        }
        if (rp == 0) st_flagged(gp.ss_ll_out + rb * 16 + t, __float_as_uint(sq), gp.flag);
      } else {
        gp.act_out[act_index(t, d0)] = h0;
        gp.act_out[act_index(t, d1)] = h1;
        if (rp == 0) gp.ss_out[rb * 16 + t] = sq;
      }
    }
  }
  }
}

// Flagged inputs of a stage (O: the attention outputs; gate/up: O's output; QKV: the previous
// down projection's output): the act blocks (3,584 16-byte units of two flagged words, 7 per
// thread) and the RMSNorm partials (448 units, if any) go to shared memory as soon as every word
// carries this layer's flag. The first round issues every load at once; later rounds reload only
// what was not ready. Only the pass's n rows are waited for (the attention writes no padding
// rows); the padding rows of the act blocks are zeros. Bounded: a timeout sets the error bit.
constexpr int MK_LL_UNITS = (int)(MK_ACT_BYTES / 8 / MK_CONS);  // act units (8 data bytes) per thread
static_assert(MK_LL_UNITS * MK_CONS * 8 == MK_ACT_BYTES, "flagged act units split evenly");
__device__ __noinline__ void mk_poll_flagged(const uint64_t* act_ll, const uint64_t* ss_ll, uint32_t F, int n,
                                             uint8_t* sAct, float* sSs, vp_state* st, volatile int* sAbort) {
  const int tid = threadIdx.x;
  const bool has_ss = ss_ll != nullptr && tid < HRB * 16 / 2;
  uint32_t pending = has_ss ? 1u << MK_LL_UNITS : 0u;
#pragma unroll
  for (int k = 0; k < MK_LL_UNITS; ++k) {
    // unit u holds data words 2u, 2u + 1 of an act block: lane (u / 2) % 32, token half u % 2
    const int u = tid + k * MK_CONS, t = (u & 1) * 8 + ((u >> 1) & 31) / 4;
    if (t < n) pending |= 1u << k;
    else reinterpret_cast<uint2*>(sAct)[u] = make_uint2(0u, 0u);
  }
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 0; pending && it < (1u << 24); ++it) {
    // every load of the round is in flight before the first check: one L2 round trip per round
    uint64_t a[MK_LL_UNITS + 1], b[MK_LL_UNITS + 1];
#pragma unroll
    for (int k = 0; k <= MK_LL_UNITS; ++k) {
      a[k] = 0;
      b[k] = 0;
      if (pending >> k & 1u)
        ld_flagged2(k < MK_LL_UNITS ? act_ll + 2 * (tid + k * MK_CONS) : ss_ll + 2 * tid, a[k], b[k]);
    }
#pragma unroll
    for (int k = 0; k < MK_LL_UNITS; ++k) {
      if ((pending >> k & 1u) && (uint32_t)(a[k] >> 32) == F && (uint32_t)(b[k] >> 32) == F) {
        reinterpret_cast<uint2*>(sAct)[tid + k * MK_CONS] = make_uint2((uint32_t)a[k], (uint32_t)b[k]);
        pending &= ~(1u << k);
      }
    }
    if ((pending >> MK_LL_UNITS & 1u) && (uint32_t)(a[MK_LL_UNITS] >> 32) == F &&
        (uint32_t)(b[MK_LL_UNITS] >> 32) == F) {
      sSs[2 * tid] = __uint_as_float((uint32_t)a[MK_LL_UNITS]);
      sSs[2 * tid + 1] = __uint_as_float((uint32_t)b[MK_LL_UNITS]);
      pending &= ~(1u << MK_LL_UNITS);
    }
    if ((it & 15) == 15 && globaltimer() - t0 > WAIT_NS) break;
  }
  if (pending) {
    set_error(st, VP_DEV_ERR_TIMEOUT);
    *sAbort = 1;
  }
}

// One GEMM stage of the pass for this CTA. piece0: global index of the stage's first piece.
// Returns false if a wait timed out.
template <int FMT, int MODE, bool DOWN = false, bool SMALL = false>
__device__ bool mk_gemm(const MegaParams& p, const GemmParams& gp, int st, int piece0, MkRing& rg,
                        uint8_t* smem, volatile int* sAbort, int cta, int G) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tid4 = lane & 3;
  uint8_t* sAct = smem + MK_OFF_ACT;
  float* sX = reinterpret_cast<float*>(smem + MK_OFF_X);
  float* sPart = reinterpret_cast<float*>(smem + MK_OFF_PART);
  float* sRs = reinterpret_cast<float*>(smem + MK_OFF_RS);
  int rb0, nrb, g0, ng;
  mk_range_g<SMALL>(st, cta, G, p.nrb_lm, rb0, nrb);
  if (nrb == 0) return true;
  mk_window(st, cta, G, g0, ng);
  const int P = mk_parts_g<SMALL>(st, nrb);
  const int tp = mk_tiles_per_slot(FMT);
  constexpr int TB = tile_bytes(FMT);
  constexpr bool down = DOWN;
  const bool dtr = gp.layer == MK_TRACE_LAYER || MODE == MODE_ARGMAX;
  (void)dtr;
  MK_CSTAMP(p, dtr, 8 * st + 0);
  // the act blocks (K = 896 stages) and the RMSNorm scale of the input rows in one round trip: the
  // act copies are in flight while the partial sums load (all 56 at once, summed in fixed order)
  // (the partials land in the partial-tile area, which is free until the jobs start)
  float* sSs = sPart;
  float* sEpc = reinterpret_cast<float*>(smem + MK_OFF_EPC);
  {
    const uint64_t pol = policy_evict_last();
    if (!down && !gp.act_ll_in)
      for (int i = threadIdx.x; i < (int)(MK_ACT_BYTES / 16); i += MK_CONS)
        cp_async16(sAct + (size_t)i * 16, reinterpret_cast<const uint4*>(gp.act) + i, 16u, pol);
    if (MODE != MODE_RESID && !gp.act_ll_in && threadIdx.x < HRB * 16 / 4)
      cp_async16(sSs + threadIdx.x * 4, gp.ss_in + threadIdx.x * 4, 16u, pol);
    cp_async_commit();
    // constants of the epilogue (QKV bias and RoPE rotations, the next RMSNorm's weights) load
    // while the copies are in flight, so the epilogue does not wait on a global round trip
    if constexpr (MODE == MODE_QKV) {  // one row-block per CTA
      const RowInfo* ri = gp.s.ri;
      const int head = rb0 >> 2, tid = threadIdx.x;
      if (tid < 16) sEpc[tid] = gp.bias[head * HD + (rb0 & 3) * 8 + (tid & 7) + (tid >> 3) * 32];
      if (head < NQ + NKV && tid >= 32 && tid < 32 + 128) {
        const int lt = tid - 32, t = lt >> 3, d = (rb0 & 3) * 8 + (lt & 7);
        if (t < ri->n)
          reinterpret_cast<float2*>(sEpc + 16)[lt] = gp.s.rope[(ri->pos + ri->depth[t]) * 32 + d];
      }
    } else if constexpr (MODE == MODE_RESID) {
      if (nrb == 1 && threadIdx.x < 16) sEpc[threadIdx.x] = gp.wnext[rb0 * 16 + threadIdx.x];
    }
    cp_async_wait<0>();
    if (gp.act_ll_in) {
      if (gp.gate) gate_wait(gp.gate, gp.gate_target, gp.s.st, sAbort);
      if (!*sAbort)
        mk_poll_flagged(gp.act_ll_in, gp.ss_ll_in, gp.flag, gp.s.ri->n, sAct, sSs, gp.s.st, sAbort);
    }
  }
  mk_sync();
  MK_CSTAMP(p, dtr, 8 * st + 1);
  // The group sums (ones-matrix MMA, one warp per K group) are handed to the tile loops through
  // an mbarrier rather than a CTA barrier, and the RMSNorm scale (read by the epilogue, after the
  // CTA barrier that ends the jobs) is formed meanwhile: neither waits for the other. The lm_head
  // folds the scale into its running argmax inside the jobs, so it keeps a CTA barrier.
  constexpr bool kGsums = !DOWN && FMT != VP_FMT_F16;
  if (MODE != MODE_RESID && warp == MK_WARPS - 1 && lane < 16)
    sRs[lane] = rms_inv([&](int r) { return sSs[r * 16 + lane]; });
  if (kGsums && warp < H / GS) {
    const uint32_t ONE2 = 0x3C003C00u;
    constexpr int NH = fmt_halves(FMT) ? 2 : 1;  // q8g32: one sum per 32-column half
    float xs[NH][2][4] = {};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint4 b = act_frag_smem(sAct, warp, j, lane);
      const int h = NH == 2 ? (j >> 1) : 0;
      mma16816(xs[h][0], ONE2, ONE2, ONE2, ONE2, b.x, b.y);
      mma16816(xs[h][1], ONE2, ONE2, ONE2, ONE2, b.z, b.w);
    }
    if (gid == 0) {
#pragma unroll
      for (int h = 0; h < NH; ++h) {
        float* xo = sX + (warp * NH + h) * 16;
        xo[2 * tid4] = xs[h][0][0];
        xo[2 * tid4 + 1] = xs[h][0][1];
        xo[8 + 2 * tid4] = xs[h][1][0];
        xo[8 + 2 * tid4 + 1] = xs[h][1][1];
      }
    }
    __syncwarp();
    if (lane == 0 && MODE != MODE_ARGMAX)
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(rg.gsum)) : "memory");
  }
  if constexpr (MODE == MODE_ARGMAX) mk_sync();
  MK_CSTAMP(p, dtr, 8 * st + 2);

  const int npieces = (nrb * ng + tp - 1) / tp;
  MkJobs J;
  J.piece0 = piece0; J.rb0 = rb0; J.nrb = nrb; J.P = P; J.ng = ng; J.actg = gp.act + (size_t)g0 * 1024;
  float* const sJobPart = sPart + (MODE == MODE_QKV || MODE == MODE_SILU ? MK_SS_SLOTS * 256 : 0);
  J.part = sJobPart;
  J.gsum = (kGsums && MODE != MODE_ARGMAX) ? rg.gsum : nullptr;
  J.gs_parity = rg.gs_phase & 1u;
#ifdef VP_TRACE_DETAIL
  J.trace = (gp.layer == MK_TRACE_LAYER || MODE == MODE_ARGMAX) ? p.trace : nullptr;
#else
  J.trace = nullptr;
#endif
  constexpr int KIND = DOWN ? JOB_DOWN : MODE == MODE_ARGMAX ? JOB_ARGMAX : JOB_SMEM;
#ifdef VP_TRACE_TWICE
  // performance experiment: the QKV jobs once more on the same data (idempotent: one piece per
  // CTA, nothing released inside), to time a warm second run
  if (MODE == MODE_QKV) {
    (void)mk_jobs<FMT, KIND>(J, rg, smem);
    MK_CSTAMP(p, dtr, 8 * st + 6);
    mk_sync();
    MK_CSTAMP(p, dtr, 8 * st + 7);
  }
#endif
  const int2 rs2 = mk_jobs<FMT, KIND>(J, rg, smem);
  bool ok = rs2.x >= 0;
  if (ok) rg.released = rs2.x;
  rg.waited = rs2.y;
  if (kGsums && MODE != MODE_ARGMAX) ++rg.gs_phase;
  MK_CSTAMP(p, dtr, 8 * st + 3);
  // this warp is done with every piece of the stage
  if (ok) ok = mk_release(rg, piece0 + npieces, lane);
  if (!ok) {
    if (lane == 0) set_error(p.s.st, VP_DEV_ERR_TIMEOUT);
    *sAbort = 1;
  }
  mk_sync();
  MK_CSTAMP(p, dtr, 8 * st + 4);
  if (*sAbort) return false;  // uniform across the CTA: every warp skips the next barrier
  if constexpr (MODE != MODE_ARGMAX) mk_epilogue<MODE, SMALL>(gp, rb0, nrb, P, sJobPart, sRs, sEpc);
  MK_CSTAMP(p, dtr, 8 * st + 5);
  return true;
}

// One pass of one request on the G CTAs of its group; this CTA is number cta of them.
template <int FMT, bool SMALL>
__device__ __forceinline__ void pass_body(const MegaParams& p, int cta, int G) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int sAbort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + MK_OFF_BAR);
  uint64_t* empty = full + MK_NSLOT;
  RowInfo* sRi = reinterpret_cast<RowInfo*>(smem + MK_OFF_RI);
  AttnSmem& sAtt = *reinterpret_cast<AttnSmem*>(smem + MK_OFF_ACT);

  if (threadIdx.x == 0) {
    for (int i = 0; i < MK_NSLOT; ++i) {
      mbar_init(full + i, 1);
      mbar_init(empty + i, MK_WARPS);
    }
    mbar_init(reinterpret_cast<uint64_t*>(smem + MK_OFF_GS), H / GS);
    fence_barrier_init();
    sAbort = 0;
  }
  cta_sync();

  if (warp == MK_WARPS) {
    mk_producer<FMT, SMALL>(p, smem, &sAbort, cta, G);
    __syncwarp();
  } else {
    unsigned long long target = 0;
    int nstamp = 0;
    auto stamp = [&]() {
      if (cta == 0 && threadIdx.x == 0 && p.trace && nstamp < MK_TRACE) p.trace[nstamp] = globaltimer();
      ++nstamp;
    };
    stamp();
    int tl = -1, tb = 0;  // layer being run (trace) and grid barriers taken in it
    auto barrier = [&]() -> bool {
      MK_CSTAMP(p, tl == MK_TRACE_LAYER, 48 + 2 * tb);
      target += (unsigned long long)G;
      const bool r = grid_barrier(p, target, &sAbort);
      MK_CSTAMP(p, tl == MK_TRACE_LAYER, 49 + 2 * tb);
      ++tb;
      stamp();
      return r;
    };

    // ---- embed the pass rows, publish RowInfo ----
    if (cta < ROWS) {
      EmbedArgs ea;
      ea.E = p.embed;
      ea.ln1 = p.ln1[0];
      ea.prompt = p.prompt;
      ea.chunk_n = p.chunk_n;
      ea.chunk_start = p.chunk_start;
      ea.total_n = p.total_n;
      embed_row<FMT>(ea, p.s, cta);
    }
    bool ok = barrier();
    if (ok) {
      const int* src = reinterpret_cast<const int*>(p.s.ri);
      int* dst = reinterpret_cast<int*>(sRi);
      for (int i = threadIdx.x; i < (int)(sizeof(RowInfo) / 4); i += MK_CONS) dst[i] = __ldcg(src + i);
    }
    // the CTA that owns row-block `cta` of the hidden dimension (O and down epilogues) keeps its
    // 16 x 16 slice of x in shared memory for the whole pass
    float* sXrb = reinterpret_cast<float*>(smem + MK_OFF_XRB);
    const bool own_x = (!SMALL || G >= H / 16) && cta < H / 16;
    if (ok && own_x)
      for (int i = threadIdx.x; i < 256; i += MK_CONS)
        sXrb[i] = __ldcg(p.s.x + (i >> 4) * H + cta * 16 + (i & 15));
    mk_sync();
    Scratch s = p.s;
    s.ri = sRi;
    const uint32_t flag0 = __ldcg(p.seq) * 64u + 1u;  // flag of layer 0 in this launch
    const bool live = ok && sRi->live != 0;
    MkRing rg;
    rg.base = smem;
    rg.full = full;
    rg.empty = empty;
    rg.released = 0;
    rg.waited = 0;
    rg.gsum = reinterpret_cast<uint64_t*>(smem + MK_OFF_GS);
    rg.gs_phase = 0;
    int piece0 = 0;
    auto pieces = [&](int st) {
      int rb0, nrb, g0, gn;
      mk_range_g<SMALL>(st, cta, G, p.nrb_lm, rb0, nrb);
      mk_window(st, cta, G, g0, gn);
      return mk_pieces(FMT, nrb, gn);
    };

    if (live) {
      // One grid barrier per layer (after gate/up): every other stage boundary is a flagged
      // transport (QKV -> attention and O -> gate/up polled directly; attention -> O and down ->
      // the next QKV gated by the producers' arrival counter). No buffer of flagged words is rewritten
      // while a reader of its previous contents is left: each is written once per layer, and its
      // next writer depends, through the layer's chain of stages, on every one of its readers.
      const int units = attn_units(sRi);
      for (int l = 0; l < p.n_layers && ok; ++l) {
        tl = l;
        tb = 0;
        MK_CSTAMP(p, l == MK_TRACE_LAYER, 56);
        const bool last = l + 1 == p.n_layers;
        GemmParams gp = {};
        gp.s = s;
        gp.layer = l;
        // QKV (+ RMSNorm scale, bias, RoPE, KV write): layer 0 reads the embed's act blocks (after
        // the embed barrier), later layers the previous down projection's flagged words
        gp.w = p.wqkv[l]; gp.act = s.act_h; gp.nrb = QKV / 16; gp.ng = H / GS;
        gp.bias = p.bqkv[l]; gp.ss_in = s.ss;
        if (l > 0) {
          gp.act_ll_in = s.dn_ll; gp.ss_ll_in = s.dn_ss_ll; gp.flag = flag0 + l - 1;
          gp.gate = p.gate + MK_GATE_DOWN; gp.gate_target = mk_gate_target(l - 1, SMALL ? min(G, HRB) : HRB);
        }
        gp.s.flag_q = flag0 + l;
        // the attention units poll the flagged q and K / V rows they need
        ok = mk_gemm<FMT, MODE_QKV, false, SMALL>(p, gp, MK_QKV, piece0, rg, smem, &sAbort, cta, G);
        piece0 += pieces(MK_QKV);
        if (!ok) break;
        s.flag_q = flag0 + l;
        // attention: each unit writes its outputs as flagged words, then arrives at the gate
        for (int u = cta; u < units; u += G) {
          MK_CSTAMP(p, l == MK_TRACE_LAYER && u == cta, 40);
#ifdef VP_TRACE_DETAIL
          attn_unit(s, l, p.max_chunks, u, sAtt,
                    (p.trace && l == MK_TRACE_LAYER && u == cta && cta < 256)
                        ? p.trace + MK_TRACE_BASE + 64 * 256 + cta : nullptr);
#else
          attn_unit(s, l, p.max_chunks, u, sAtt);
#endif
          if (threadIdx.x == 0) gate_arrive(p.gate + MK_GATE_ATT);
          MK_CSTAMP(p, l == MK_TRACE_LAYER && u == cta, 42);
        }
        // O + residual: polls the attention outputs once every unit arrived
        gp = GemmParams{};
        gp.s = s; gp.layer = l;
        gp.w = p.wo[l]; gp.nrb = H / 16; gp.ng = H / GS;
        gp.act_ll_in = s.att_ll; gp.flag = flag0 + l;
        gp.gate = p.gate + MK_GATE_ATT; gp.gate_target = mk_gate_target(l, units);
        gp.wnext = p.ln2[l];
        gp.act_ll_out = s.act_ll; gp.ss_ll_out = s.ss_ll;
        gp.xs = own_x ? sXrb : nullptr;
        ok = mk_gemm<FMT, MODE_RESID, false, SMALL>(p, gp, MK_O, piece0, rg, smem, &sAbort, cta, G);
        piece0 += pieces(MK_O);
        if (!ok) break;
        // gate/up + SiLU: polls O's outputs directly (no gate: the O stage is short, and the
        // polls start as its CTAs finish their part)
        gp = GemmParams{};
        gp.s = s; gp.layer = l;
        gp.w = p.wgu[l]; gp.nrb = 2 * F / 16; gp.ng = H / GS;
        gp.act_ll_in = s.act_ll; gp.ss_ll_in = s.ss_ll; gp.flag = flag0 + l; gp.act_out = s.act_f;
        ok = mk_gemm<FMT, MODE_SILU, false, SMALL>(p, gp, MK_GU, piece0, rg, smem, &sAbort, cta, G) && barrier();
        piece0 += pieces(MK_GU);
        if (!ok) break;
        // down + residual: flagged words for the next QKV; the last layer's output feeds the
        // lm_head through plain act blocks and a grid barrier
        gp = GemmParams{};
        gp.s = s; gp.layer = l;
        gp.w = p.wd[l]; gp.act = s.act_f; gp.nrb = H / 16; gp.ng = F / GS;
        gp.wnext = last ? p.final_norm : p.ln1[l + 1];
        const bool to_lm = last && p.do_lm;
        gp.flag = flag0 + l;
        if (to_lm) {
          gp.ss_out = s.ss; gp.act_out = s.act_h;
        } else {
          gp.act_ll_out = s.dn_ll; gp.ss_ll_out = s.dn_ss_ll;
        }
        if (mk_down_split(G)) {
          if (own_x) gp.part_ll_in = s.dnp_ll;
          else gp.part_ll_out = s.dnp_ll;
        }
        gp.xs = own_x ? sXrb : nullptr;
        ok = mk_gemm<FMT, MODE_RESID, true, SMALL>(p, gp, MK_DOWN, piece0, rg, smem, &sAbort, cta, G);
        piece0 += pieces(MK_DOWN);
        if (!ok) break;
        if (to_lm) {
          ok = barrier();
        } else if (cta < (SMALL ? min(G, HRB) : HRB)) {  // the down CTAs (the owners of split row-blocks)
          mk_sync();
          if (threadIdx.x == 0) gate_arrive(p.gate + MK_GATE_DOWN);
        }
      }
      if (ok && p.do_lm) {
        GemmParams gp = {};
        gp.s = s;
        gp.w = p.embed; gp.act = s.act_h; gp.nrb = p.nrb_lm; gp.ng = H / GS; gp.ss_in = s.ss;
        if (lane < 16) {  // every warp's running best starts empty
          reinterpret_cast<float*>(smem + MK_OFF_LMV)[warp * 16 + lane] = -INFINITY;
          reinterpret_cast<int*>(smem + MK_OFF_LMI)[warp * 16 + lane] = 0x7fffffff;
        }
        ok = mk_gemm<FMT, MODE_ARGMAX, false, SMALL>(p, gp, MK_LM, piece0, rg, smem, &sAbort, cta, G);
        // per-CTA best per token from the warps' running bests
        float* sLmV = reinterpret_cast<float*>(smem + MK_OFF_LMV);
        int* sLmI = reinterpret_cast<int*>(smem + MK_OFF_LMI);
        mk_sync();
        if (threadIdx.x < 16) {
          const int t = threadIdx.x;
          float bv = sLmV[t];
          int bi = sLmI[t];
          for (int w = 1; w < MK_WARPS; ++w) {
            const float v = sLmV[w * 16 + t];
            const int id = sLmI[w * 16 + t];
            if (v > bv || (v == bv && id < bi)) { bv = v; bi = id; }
          }
          p.lm_pval[t * G + cta] = bv;
          p.lm_pidx[t * G + cta] = bi;
        }
        ok = ok && barrier();
        if (ok && p.do_commit && cta == 0) commit_body(s, p.lm_pval, p.lm_pidx, G);
      }
    }
    if (!live || !ok) sAbort = 1;  // the producer stops waiting for releases
    stamp();
  }
  cta_sync();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(p.exit_ctr, 1u) == (unsigned)G - 1) {
      *p.bar = 0ull;  // every CTA is past its last barrier: the next launch starts from zero
      for (int i = 0; i < MK_GATES; ++i) p.gate[i] = 0u;
      *p.exit_ctr = 0u;
      *p.seq = *p.seq + 1u;  // the next launch's flags differ from every word written here
      __threadfence();
    }
  }
}

// One verify pass (or prefill chunk) of one request on every CTA of the launch.
template <int FMT>
__global__ void __launch_bounds__(MK_THREADS, 1) k_pass(const __grid_constant__ MegaParams p) {
  pass_body<FMT, false>(p, blockIdx.x, gridDim.x);
}

// Passes of up to MK_MAX_GROUPS requests in one launch, each on its own contiguous group of
// gridDim.x / groups CTAs with its own context (barrier counters, state, scratch, KV cache): a
// single pass is bound by the latency of its dependent stages, not by the SMs or HBM, so more
// requests on shares of the SMs cost little time each. SMALL: groups of fewer than 72 CTAs.
constexpr int MK_MAX_GROUPS = 4;
struct BatchParams {
  MegaParams p[MK_MAX_GROUPS];
  int groups;
};
// a __grid_constant__ parameter block above the classic 4 KB: CUDA 12.1+ takes up to 32,764 bytes
static_assert(sizeof(BatchParams) <= 32764, "kernel parameter block");
template <int FMT, bool SMALL>
__global__ void __launch_bounds__(MK_THREADS, 1) k_pass_groups(const __grid_constant__ BatchParams bp) {
  const int per = gridDim.x / bp.groups, g = blockIdx.x / per;
  pass_body<FMT, SMALL>(bp.p[g], blockIdx.x - g * per, per);
}

}  // namespace vp
