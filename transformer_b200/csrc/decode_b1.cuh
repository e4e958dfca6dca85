// decode_b1.cuh — persistent single-sequence decode megakernel (sm_100a).
//
// One launch runs a whole decode step of the decoder: embedding -> L layers of
// [RMSNorm, QKV GEMV, RoPE, GQA attention over the KV cache, O GEMV + residual,
// RMSNorm, gate/up GEMV + SwiGLU, down GEMV + residual] -> final RMSNorm ->
// tied-embedding logits -> argmax.  It replaces the reference's Triton kernel
// `_multi_sm_decode` (kernels/multi_sm_decode.py:35-357) and follows its math
// (RMSNorm :121-126, QKV :133-152, RoPE :154-173, attention :182-221 with the
// new position's K/V used in f32 as at :197/:205, O-proj :223-232, SwiGLU
// :270-291, logits + first-index argmax :314-357).
//
// Structure (B200-first, not a translation):
//  * grid = one CTA per SM (cooperative launch, so co-residency is checked at
//    launch), 8 consumer warps + 1 producer warp.
//  * Every GEMV's output rows are split evenly over the CTAs.  The weights are
//    packed output-row-major, so a CTA's rows for a phase are one contiguous
//    byte range.  The producer warp streams the CTA's ranges for the whole step
//    (all layers, then the logits rows) through a ring of shared-memory stages
//    with `cp.async.bulk` + mbarriers and an L2 evict-first hint.  It never
//    waits on activations, so HBM streaming continues while consumers wait.
//  * Consumers exchange activations through 8-byte words in global memory
//    (payload + launch flag, see b2d_ptx.cuh): each producer of a value writes
//    it with one store; every reader polls the words it needs.  No grid-wide
//    barrier and no memset per step: the flag changes every launch.
//  * Every wait is bounded (global timer); a timeout sets the workspace status
//    word and an abort marker and all CTAs leave.  A CTA never exits with its
//    own bulk copies in flight.
//  * All reductions run in a fixed order (no float atomics): bit-reproducible.
#pragma once

#include <cstddef>

#include "b2d_ptx.cuh"

namespace b2d {

// Device status word (Control::status).  0 = ok.
enum : uint32_t {
  ST_TIMEOUT = 0x100u,    // | site
  ST_BAD_INPUT = 0x200u,  // | 1 token, 2 pos
};
enum : uint32_t {
  SITE_H = 1, SITE_QKV = 2, SITE_ATT = 3, SITE_HM = 4, SITE_ACT = 5, SITE_FINAL = 6,
  SITE_FULL = 7, SITE_EMPTY = 8, SITE_DRAIN = 9, SITE_VATT = 10, SITE_TOKEN = 11,
};

struct Control {  // each word on its own 128-byte line
  uint32_t status;
  uint32_t pad0[31];
  uint32_t gen;
  uint32_t pad1[31];
  uint32_t arrive;
  uint32_t pad2[31];
  uint32_t abort_flag;
  uint32_t pad3[31];
  uint64_t tok_word;  // multi-step launches: (step flag << 32) | token of the step just finished
  uint32_t pad4[30];
};

struct DecodeArgs {
  const uint8_t* wbase;  // packed weights (see include/b2d.h layout)
  uint64_t layer_stride, off_qkv, off_o, off_gu, off_down, off_emb;
  const float* ln1;  // [L][D]
  const float* ln2;  // [L][D]
  const float* lnf;  // [D]
  const float* rcos; // [ctx][DH/2]
  const float* rsin;
  const int32_t* tok;  // device token, or null: then tok_val
  const int32_t* pos;  // device position, or null: then pos_val
  int32_t tok_val, pos_val;  // the first step's token and position passed by value
  __nv_bfloat16* kv;  // [L][2][NKV][ctx][DH]
  float* logits;      // [V] or null
  int32_t* next_tok;
  int n_steps;        // greedy tokens per launch (>= 1): step s decodes at pos + s
  int32_t* tok_out;   // [n_steps] the token of every step, or null
  uint64_t* words;    // exchange words
  uint64_t* acc;      // cluster kernel: residual accumulators [2 parities][2 n_layers][D]
  Control* ctl;
  float* am_val;      // [grid]
  int32_t* am_idx;
  uint32_t layer_words;                   // exchange words per layer
  uint32_t w_att, w_hm, w_act;            // word offsets in a layer (H at 0, QKV at D)
  int vocab, n_layers, ctx;
  int att_T;          // KV positions per attention unit (multiple of 64)
  int grid_part;      // CTAs the work is split over (== gridDim.x except in fault tests)
  uint64_t wait_ns;   // bound on every wait
  float eps;
  uint64_t* trace;    // optional per-CTA phase stamps (global timer, ns), or null
  int trace_stride;   // stamps per CTA
  uint32_t poll_ns;   // back-off between failed polls (0 = spin)
  int max_inflight;   // bulk copies in flight per CTA (<= kStages)
  // diagnostics: per-CTA stage stamps [3][stage_stride] (copy issued by the
  // producer; stage seen full by consumer warp 0; warp 0 done with it), or null
  uint64_t* stage_trace;
  int stage_stride;
};

// Phase-stamp slots (per CTA): 0 = start, then per layer kTracePerLayer
// stamps, then final gather / logits / end.  Stamps exist only in the kernel
// instantiated with TR = true (launched when a trace buffer is set), so the
// production kernel carries no diagnostic branches.
constexpr int kTracePerLayer = 13;
template <bool TR>
__device__ __forceinline__ void trace_stamp(const DecodeArgs& A, int slot) {
  if constexpr (TR) {
    if (A.trace != nullptr && threadIdx.x == 0 && slot < A.trace_stride)
      A.trace[static_cast<size_t>(blockIdx.x) * A.trace_stride + slot] = globaltimer_ns();
  }
}
// Weight-stage stamps (kind 0 issued, 1 seen full, 2 consumed), TR only.
template <bool TR>
__device__ __forceinline__ void stage_stamp(const DecodeArgs& A, int cta, int kind, uint32_t seq) {
  if constexpr (TR) {
    if (A.stage_trace != nullptr && seq < static_cast<uint32_t>(A.stage_stride))
      A.stage_trace[(static_cast<size_t>(cta) * 3 + kind) * A.stage_stride + seq] = globaltimer_ns();
  }
}

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
// A stage holds whole weight rows at a pitch of the row plus 16 bytes (pitch =
// 16 mod 128), so the 8 rows an ldmatrix reads fall in distinct banks.
constexpr int kRowPad = 16;
// 8 rows of 2 KB or 3 rows of 5.5 KB, padded (306M shapes); a multiple of
// 1024 so that stages can take 128-byte-swizzled tensor copies
constexpr int kStageBytes = 17408;
constexpr int kStages = 10;
constexpr int kAttWords = 66;       // per attention unit: o[64], m, l
constexpr int kMaxSplits = 4;       // attention units per head
constexpr int kMinGrid = 128;       // fewest CTAs the phase register budgets assume
// GEMV phases of a step, in streaming order (Smem::rng index / 2)
enum Phase : int { PH_QKV = 0, PH_O = 1, PH_GU = 2, PH_DOWN = 3, PH_VOCAB = 4, kPhases = 5 };

template <int D_, int DFF_, int NH_, int NKV_>
struct Shape {
  static constexpr int D = D_, DFF = DFF_, NH = NH_, NKV = NKV_, DH = 64;
  static constexpr int GQA = NH / NKV;
  static constexpr int QKV = (NH + 2 * NKV) * DH;
  static constexpr int KD = D / 256;    // 16-byte chunks per lane along K = D
  static constexpr int KF = DFF / 256;  // along K = DFF
  static constexpr int ROWB_D = 2 * D;
  static constexpr int ROWB_F = 2 * DFF;
  static constexpr int PITCH_D = ROWB_D + kRowPad, PITCH_F = ROWB_F + kRowPad;
  static constexpr int RPS_D = kStageBytes / PITCH_D;       // rows of K=D per stage
  static constexpr int RPS_F = kStageBytes / PITCH_F;       // down rows per stage
  // 16-row MMA tiles per CTA of each layer phase (grids of >= kMinGrid CTAs)
  static constexpr int tiles_for(int rows) { return ((rows + kMinGrid - 1) / kMinGrid + 15) / 16; }
  static constexpr int MT_QKV = tiles_for(QKV), MT_O = tiles_for(D), MT_DOWN = tiles_for(D);
  static constexpr int MT_GU = (4 * ((DFF / 2 + kMinGrid - 1) / kMinGrid) + 15) / 16;
  static constexpr int MT_MAX = MT_GU > MT_QKV ? MT_GU : MT_QKV;
  static_assert(D % 128 == 0 && DFF % 128 == 0, "K splits into 8 warp slices of whole 16-column steps");
  static_assert(PITCH_D % 128 == 16 && PITCH_F % 128 == 16, "padded row pitch");
  static constexpr int XMAX = DFF > D ? DFF : D;
  // gate/up rows per CTA: the DFF / 2 act words (2 pairs = 4 rows each) split over >= kMinGrid CTAs
  static constexpr int GU_ROWS_MAX = 4 * ((DFF / 2 + kMinGrid - 1) / kMinGrid);
  static_assert(GU_ROWS_MAX <= 16 * ((4 * ((DFF / 2 + kMinGrid - 1) / kMinGrid) + 15) / 16), "gate/up tiles");
  static constexpr int NP_D = (D / 2 + kConsumers - 1) / kConsumers;        // residual word pairs per thread
  static constexpr int NP_ACT = (DFF / 4 + kConsumers - 1) / kConsumers;    // act word pairs per thread
  static_assert(DFF % 4 == 0, "act words hold two bf16 values, read in pairs");
  static_assert(D % 256 == 0 && DFF % 256 == 0, "row length must be a multiple of 256");
  static_assert(RPS_D >= 1 && RPS_F >= 1, "stage too small");
  static_assert(NH % NKV == 0, "GQA");
  static_assert(NH * 16 <= kConsumers, "attention merge uses 16 threads per head");
  static_assert(NH * kMaxSplits <= kConsumers, "one thread per attention unit in the merge");
};

// Shared-memory carve-up (dynamic).
template <class S>
struct Smem {
  alignas(128) uint8_t stage[kStages][kStageBytes];
  uint64_t full[kStages];
  uint64_t empty[kStages];
  float h[S::D];          // residual stream (f32)
  alignas(16) __nv_bfloat16 xb[S::XMAX];  // GEMV input vector (bf16, natural order)
  alignas(128) __nv_bfloat16 katt[128][64];  // K rows of the attention unit's pass
  alignas(128) __nv_bfloat16 vatt[128][64];  // V rows of the attention unit's pass
  uint64_t att_bar;       // completes the K/V staging copies
  float qkv[3 * 64];      // attention unit inputs
  alignas(16) float rq[64];  // post-RoPE q (pre-scaled); read as float4
  alignas(16) float rk[64];  // post-RoPE k
  float wm[kConsumerWarps], wl[kConsumerWarps];
  float wo[kConsumerWarps][64];
  float red[kConsumerWarps];
  float ml[2 * kConsumers];  // (m, l) of each attention unit
  float am_v[kConsumerWarps];
  int am_i[kConsumerWarps];
  alignas(16) float gu_out[S::GU_ROWS_MAX];  // this CTA's gate/up dot products (gate j, up j, ...)
  float part[kConsumerWarps][S::MT_MAX * 16];  // GEMV: each warp's K-slice partial of every row
  int rng[2 * kPhases];                      // this CTA's unit range [a, b) of each GEMV phase
  int abort;
  int tok_in;  // multi-step: this step's input token
};

// Fields read with 16-byte vector loads or written by bulk copies.
template <class S>
struct SmemChecks {
  static_assert(offsetof(Smem<S>, stage) % 128 == 0, "stage alignment");
  static_assert(kStageBytes % 16 == 0, "stage size");
  static_assert(offsetof(Smem<S>, xb) % 16 == 0, "xb alignment");
  static_assert(offsetof(Smem<S>, vatt) % 128 == 0 && offsetof(Smem<S>, katt) % 128 == 0, "K/V staging alignment");
  static_assert(offsetof(Smem<S>, rq) % 16 == 0, "rq alignment");
  static_assert(offsetof(Smem<S>, gu_out) % 16 == 0, "gu_out alignment (read as float4)");
  static_assert(offsetof(Smem<S>, full) % 8 == 0 && offsetof(Smem<S>, att_bar) % 8 == 0, "mbarrier alignment");
  static_assert(sizeof(Smem<S>) <= 232448, "shared memory per CTA");
  static constexpr bool ok = true;
};

__device__ __forceinline__ int split_begin(int c, int n, int g) {
  return static_cast<int>((static_cast<long long>(c) * n) / g);
}

// Raise a device error once (first error wins) and mark this launch aborted.
__device__ __forceinline__ void raise_error(Control* ctl, uint32_t code, uint32_t flag) {
  atomicCAS(&ctl->status, 0u, code);
  st_relaxed_u32(&ctl->abort_flag, flag);
}

// True when the wait must give up (time limit reached or another CTA aborted).
__device__ __forceinline__ bool wait_expired(const DecodeArgs& A, uint32_t flag, uint64_t t0,
                                             uint32_t site) {
  if (ld_relaxed_u32(&A.ctl->abort_flag) == flag) return true;
  if (globaltimer_ns() - t0 > A.wait_ns) {
    raise_error(A.ctl, ST_TIMEOUT | site, flag);
    return true;
  }
  return false;
}

// Bounded-wait bookkeeping that stays off the critical path: the clock is
// read every 128 polls and the abort marker (a global load) only once a wait
// has already lasted 20 us, which normal waits never reach.
struct Waiter {
  uint64_t start = 0;
  uint32_t spins = 0;
  __device__ __forceinline__ bool expired(const DecodeArgs& A, uint32_t flag, uint64_t t0, uint32_t site) {
    if ((++spins & 127u) != 0) return false;
    const uint64_t now = globaltimer_ns();
    if (start == 0) { start = now; return false; }
    if (now - start < 20000u) return false;
    return wait_expired(A, flag, t0, site);
  }
};

// The same bookkeeping with the clock check out of line, so that a wait site
// keeps only the poll counter inline.  Returns the wait's start time (set by
// the first check), or 0 when the wait must give up; every site using it
// stops waiting once expired() returns true.  The cluster kernel's producer
// warp uses it: its poll loops stay small, and it issues the weight stream
// faster (measured: config 1 263.4 -> 236.8 us/token, config 2 271.6 ->
// 269.5 us/token).  The consumers' waits keep the inline form, which measured
// the same or faster there.
__device__ __noinline__ uint64_t waiter_check(uint64_t start, Control* ctl, uint64_t wait_ns, uint32_t flag,
                                              uint64_t t0, uint32_t site) {
  const uint64_t now = globaltimer_ns();
  if (start == 0) return now;
  if (now - start < 20000u) return start;
  if (ld_relaxed_u32(&ctl->abort_flag) == flag) return 0;
  if (now - t0 > wait_ns) {
    raise_error(ctl, ST_TIMEOUT | site, flag);
    return 0;
  }
  return start;
}
struct ProducerWaiter {
  uint64_t start = 0;
  uint32_t spins = 0;
  __device__ __forceinline__ bool expired(const DecodeArgs& A, uint32_t flag, uint64_t t0, uint32_t site) {
    if ((++spins & 127u) != 0) return false;
    start = waiter_check(start, A.ctl, A.wait_ns, flag, t0, site);
    return start == 0;
  }
};

// Gather up to N word pairs per thread.  addr(i) -> pointer to pair i (16-B
// aligned); valid(i) says whether this thread owns item i; store(i, a, b)
// receives the payloads.  All owned loads are issued together, then the
// thread spins on one pending pair at a time.  Returns false on timeout/abort.
template <int N, int GRP = 8, class AddrF, class ValidF, class StoreF>
__device__ __forceinline__ bool gather_pairs(const DecodeArgs& A, uint32_t flag, uint64_t t0,
                                             uint32_t site, AddrF addr, ValidF valid, StoreF store) {
  static_assert(N <= 32, "pending mask is 32 bits");  // GRP: loads issued together per thread
  uint32_t pending = 0;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (valid(i)) pending |= 1u << i;
  Waiter wt;
  while (pending) {
#pragma unroll
    for (int g = 0; g < N; g += GRP) {
      uint64_t a[GRP], b[GRP];
#pragma unroll
      for (int k = 0; k < GRP; ++k)
        if (g + k < N && (pending & (1u << (g + k)))) ld_words2(addr(g + k), a[k], b[k]);
#pragma unroll
      for (int k = 0; k < GRP; ++k) {
        const int i = g + k;
        if (i < N && (pending & (1u << i)) && word_flag(a[k]) == flag && word_flag(b[k]) == flag) {
          store(i, word_val(a[k]), word_val(b[k]));
          pending &= ~(1u << i);
        }
      }
    }
    if (!pending) break;
    // Spin on one pending pair, then re-check everything still pending.
    const int i0 = __ffs(pending) - 1;
    const uint64_t* p0 = nullptr;
#pragma unroll
    for (int i = 0; i < N; ++i)
      if (i == i0) p0 = addr(i);
    while (true) {
      uint64_t x, y;
      ld_words2(p0, x, y);
      if (word_flag(x) == flag && word_flag(y) == flag) break;
      if (A.poll_ns) __nanosleep(A.poll_ns);
      if (wt.expired(A, flag, t0, site)) return false;
    }
  }
  return true;
}

// Consumer-side view of a stage ring of NS stages of SB bytes.
template <int NS, int SB>
struct RingT {
  static constexpr int kN = NS;
  uint8_t (*stage)[SB];
  uint64_t* full;
  uint64_t* empty;
  uint32_t seq;
};
using Ring = RingT<kStages, kStageBytes>;

// Warp-uniform: every lane acquires the stage itself; lane 0 decides timeouts.
template <class R>
__device__ __forceinline__ bool wait_full(const DecodeArgs& A, R& r, uint32_t flag, uint64_t t0) {
  const uint32_t slot = r.seq % R::kN, par = (r.seq / R::kN) & 1u;
  const int lane = threadIdx.x & 31;
  Waiter wt;
  while (true) {
    const bool done = mbar_test(&r.full[slot], par);
    if (__all_sync(0xffffffffu, done)) return true;
    const bool exp = lane == 0 ? wt.expired(A, flag, t0, SITE_FULL) : false;
    if (__shfl_sync(0xffffffffu, exp ? 1 : 0, 0)) return false;
  }
}

// Warp-uniform: waits until the n stages ring.seq .. ring.seq+n-1 (n <=
// kStages / 2) have landed.  Lane i tests stage seq+i, so a phase whose
// stages are already resident (the usual case: the producer runs ~20 us
// ahead) costs one barrier round trip instead of one per stage; __syncwarp
// then orders every lane after the acquiring lanes.
template <class R>
__device__ __forceinline__ bool wait_full_n(const DecodeArgs& A, R& r, int n, uint32_t flag, uint64_t t0) {
  const int lane = threadIdx.x & 31;
  const uint32_t sq = r.seq + static_cast<uint32_t>(lane);
  Waiter wt;
  while (true) {
    const bool done = lane >= n || mbar_test(&r.full[sq % R::kN], (sq / R::kN) & 1u);
    if (__all_sync(0xffffffffu, done)) break;
    const bool exp = lane == 0 ? wt.expired(A, flag, t0, SITE_FULL) : false;
    if (__shfl_sync(0xffffffffu, exp ? 1 : 0, 0)) return false;
  }
  __syncwarp();
  return true;
}

// Warp-uniform: this warp is done with stages seq .. seq+n-1 (lane i arrives
// on stage seq+i's empty barrier).
template <class R>
__device__ __forceinline__ void release_n(R& r, int n) {
  const int lane = threadIdx.x & 31;
  __syncwarp();
  if (lane < n) mbar_arrive(&r.empty[(r.seq + static_cast<uint32_t>(lane)) % R::kN]);
  r.seq += static_cast<uint32_t>(n);
}


// The GEMV input vector, read from Smem::xb (bf16, natural order).  Lane l
// multiplies weight elements k*256 + l*8 + j (k < KI, j < 8), i.e. the 16-byte
// chunk k*32 + l of the vector: one conflict-free 16-byte read per lane and K
// step serves every row of the warp's units (the K loop is outermost).  The
// unpacked bf16 pairs are exact f32 values.
struct X4 {
  uint64_t q[4];
};
struct XSmem {
  const uint4* p;
  __device__ __forceinline__ X4 chunk(int k) const {
    const uint4 u = p[k * 32 + (threadIdx.x & 31)];
    return X4{{bf2pack(u.x), bf2pack(u.y), bf2pack(u.z), bf2pack(u.w)}};
  }
};

// acc += 8 bf16 weights (w) x the lane's 8 activations of one chunk.
__device__ __forceinline__ void dot8r(const uint4 w, const X4& x, uint64_t& a0, uint64_t& a1) {
  a0 = ffma2(bf2pack(w.x), x.q[0], a0);
  a1 = ffma2(bf2pack(w.y), x.q[1], a1);
  a0 = ffma2(bf2pack(w.z), x.q[2], a0);
  a1 = ffma2(bf2pack(w.w), x.q[3], a1);
}

// One GEMV phase over this CTA's rows [u_begin, u_end) on warp-level tensor-core
// MMAs (mma.m16n8k16, bf16 in, f32 accumulate).  All of the phase's stages are
// resident at once (at most kStages); warp w takes the K slice [w K/8,
// (w+1) K/8) of every 16-row tile: A = 16 weight rows (ldmatrix; rows past
// u_end read a valid row and are ignored), B = the input vector in all 8
// columns (two 32-bit shared reads per step, so every output column is the
// dot product).  The warps' partials of each row meet in `part` (PSTRIDE
// floats per warp) and thread r sums them in warp order (deterministic), then
// calls out(u_begin + r, v).  Ends with the phase's closing barrier; returns
// the AND of every warp's waits.
template <int K, int PITCH, int PS, int MT, int PSTRIDE, bool TR, class Out>
__device__ __forceinline__ bool gemv_phase(const DecodeArgs& A, Ring& ring, float* part, const __nv_bfloat16* xb,
                                           uint32_t flag, uint64_t t0, int u_begin, int u_end, Out out) {
  static_assert(MT * 16 <= PSTRIDE, "partial buffer");
  constexpr int KS = K / 16 / kConsumerWarps;  // 16-column steps per warp
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int rows = u_end - u_begin;
  const int ns = rows > 0 ? (rows + PS - 1) / PS : 0;
  bool ok = rows <= MT * 16 && ns <= kStages;
  if (ok && ns > 0) ok = wait_full_n(A, ring, ns, flag, t0);
  if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 1, ring.seq);
  if (ok && rows > 0) {
    // ldmatrix.x4 rows: lane l gives row (l & 7) + 8 ((l >> 3) & 1) of the tile, columns + 8 (l >> 4)
    const int lr = (lane & 7) + 8 * ((lane >> 3) & 1), lk = 8 * (lane >> 4);
    uint32_t rbase[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int r = min(mt * 16 + lr, rows - 1);  // rows past the range: any valid row
      const int st = r / PS;
      rbase[mt] = smem_addr(ring.stage[(ring.seq + static_cast<uint32_t>(st)) % kStages]) +
                  static_cast<uint32_t>((r - st * PS) * PITCH + 2 * lk);
    }
    // two accumulator chains (even / odd steps) so consecutive MMAs do not wait on each other
    float acc[2][MT][4];
#pragma unroll
    for (int c = 0; c < 2; ++c)
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) acc[c][mt][0] = acc[c][mt][1] = acc[c][mt][2] = acc[c][mt][3] = 0.f;
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(xb);
    const int k0 = warp * KS * 16;
#pragma unroll 4
    for (int s = 0; s < KS; ++s) {
      const int k = k0 + 16 * s;
      const uint32_t b0 = x32[(k + 2 * tig) >> 1], b1 = x32[(k + 8 + 2 * tig) >> 1];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4(rbase[mt] + 2u * static_cast<uint32_t>(k), a0, a1, a2, a3);
        mma_bf16(acc[s & 1][mt], a0, a1, a2, a3, b0, b1);
      }
    }
    if (tig == 0) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        part[warp * PSTRIDE + mt * 16 + gid] = acc[0][mt][0] + acc[1][mt][0];      // row gid of the tile
        part[warp * PSTRIDE + mt * 16 + gid + 8] = acc[0][mt][2] + acc[1][mt][2];  // row gid + 8
      }
    }
  }
  if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 2, ring.seq);
  if (ok) release_n(ring, ns);
  ok = consumer_sync_and<kConsumers>(ok);
  if (!ok) return false;
  if (t < rows) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) v += part[w * PSTRIDE + t];
    out(u_begin + t, v);
  }
  return true;
}

// Same streaming for many units per warp (the logits): reduce per stage.
template <int KI, int PITCH, int PS, class R, int GROUP = R::kN / 2, bool TR = false, class Out>
__device__ __forceinline__ bool gemv_phase_wide(const DecodeArgs& A, R& ring, uint32_t flag, uint64_t t0,
                                                int u_begin, int u_end, const XSmem x, Out out) {
  constexpr int kGroupStages = GROUP;  // stages waited for (and released) together
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  bool ok = true;
  for (int g0 = u_begin; g0 < u_end && ok; g0 += kGroupStages * PS) {
    const int g1 = min(g0 + kGroupStages * PS, u_end);
    const int ns = (g1 - g0 + PS - 1) / PS;
    ok = wait_full_n(A, ring, ns, flag, t0);
    if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 1, ring.seq);
    if (ok) {
      const int first = g0 + ((warp - (g0 - u_begin)) % kConsumerWarps + kConsumerWarps) % kConsumerWarps;
      for (int u = first; u < g1; u += kConsumerWarps) {
        const int st = (u - g0) / PS;
        const uint8_t* sb = ring.stage[(ring.seq + static_cast<uint32_t>(st)) % R::kN];
        const uint4* rp = reinterpret_cast<const uint4*>(sb + static_cast<size_t>(u - g0 - st * PS) * PITCH);
        uint64_t a0 = 0ull, a1 = 0ull;
#pragma unroll
        for (int k = 0; k < KI; ++k) dot8r(rp[k * 32 + lane], x.chunk(k), a0, a1);
        out(u, warp_sum(f2sum(a0) + f2sum(a1)), 0.f);
      }
    }
    if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 2, ring.seq);
    release_n(ring, ns);
  }
  return ok;
}

// Residual stream -> GEMV input: thread t holds the residual pairs
// (elements 2k, 2k + 1, k = t + 256 i, i < NP) in hv.  Stores them into sm.h,
// then x = bf16(h * rsqrt(mean(h^2) + eps) * g) into sm.xb (RMSNorm,
// reference :121-126); the sum of squares is taken from the registers, so one
// barrier publishes h and the per-warp sums together.  `ok` enters the
// barrier's AND; returns the combined flag.
template <class S, int NP>
__device__ __forceinline__ bool norm_pairs(Smem<S>& sm, const float (&hv)[NP][2], const float2 (&g)[NP],
                                           float eps, bool ok) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int k = t + i * kConsumers;
    if (k < S::D / 2) {
      sm.h[2 * k] = hv[i][0];
      sm.h[2 * k + 1] = hv[i][1];
      ss = fmaf(hv[i][0], hv[i][0], ss);
      ss = fmaf(hv[i][1], hv[i][1], ss);
    }
  }
  ss = warp_sum(ss);
  if (lane == 0) sm.red[warp] = ss;
  ok = consumer_sync_and<kConsumers>(ok);
  if (!ok) return false;
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) tot += sm.red[w];
  const float r = rsqrtf(tot / static_cast<float>(S::D) + eps);
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int k = t + i * kConsumers;
    if (k < S::D / 2)
      reinterpret_cast<__nv_bfloat162*>(sm.xb)[k] = __floats2bfloat162_rn(hv[i][0] * r * g[i].x, hv[i][1] * r * g[i].y);
  }
  consumer_sync<kConsumers>();
  return true;
}

// Norm gains of this thread's residual pairs (loaded ahead of the wait that
// precedes the norm, so their latency is hidden).
template <class S, int NP>
__device__ __forceinline__ void load_gain_pairs(const float* gain, float2 (&g)[NP]) {
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    const int k = threadIdx.x + i * kConsumers;
    g[i] = k < S::D / 2 ? __ldg(reinterpret_cast<const float2*>(gain) + k) : make_float2(0.f, 0.f);
  }
}

// Gathers the residual stream (D f32 words at `src`, written by other CTAs)
// and normalises it into sm.xb with gains `gain`.
template <class S>
__device__ __forceinline__ bool gather_norm(const DecodeArgs& A, Smem<S>& sm, const uint64_t* src, uint32_t flag,
                                            uint64_t t0, uint32_t site, const float* gain) {
  constexpr int NP = S::NP_D;
  const int t = threadIdx.x;
  float2 g[NP];
  load_gain_pairs<S, NP>(gain, g);
  float hv[NP][2];
#pragma unroll
  for (int i = 0; i < NP; ++i) hv[i][0] = hv[i][1] = 0.f;
  const bool ok = gather_pairs<NP>(
      A, flag, t0, site, [&](int i) { return src + 2 * (t + i * kConsumers); },
      [&](int i) { return t + i * kConsumers < S::D / 2; },
      [&](int i, float a, float b) { hv[i][0] = a; hv[i][1] = b; });
  return norm_pairs<S, NP>(sm, hv, g, A.eps, ok);
}

// Producer: streams this CTA's weight ranges for the whole step.
template <class S, bool TR>
// The whole producer warp runs it: lane 0 waits for ring slots and arms the
// stages; the rows of a padded stage are copied by lanes 0..rows-1 in parallel.
__device__ void producer_loop(const DecodeArgs& A, Smem<S>& sm, int cta, uint32_t flag, uint64_t t0, int nsteps) {
  const int lane = threadIdx.x & 31;
  const uint64_t pol = l2_policy_evict_first();
  const int G = A.grid_part;
  uint32_t seq = 0;
  bool ok = true;
  // Copies are capped at max_inflight per CTA: enough to keep HBM busy, few
  // enough that the memory queues stay short for the latency-critical
  // exchange words.  Landed stages still accumulate in the ring.
  uint32_t landed = 0;
  const uint32_t cap = static_cast<uint32_t>(A.max_inflight);
  // one stage: `cnt` rows of `rb` bytes each, from consecutive rows at src
  auto issue = [&](const uint8_t* src, int cnt, uint32_t rb, uint32_t pitch) {
    const uint32_t slot = seq % kStages;
    bool good = true;
    if (lane == 0) {
      while (good && seq - landed >= cap) {
        Waiter wt;
        while (!mbar_test(&sm.full[landed % kStages], (landed / kStages) & 1u)) {
          if ((*reinterpret_cast<volatile int*>(&sm.abort) || wt.expired(A, flag, t0, SITE_FULL))) {
            good = false;
            break;
          }
        }
        if (good) ++landed;
      }
      if (good && seq >= kStages) {
        const uint32_t par = ((seq / kStages) - 1) & 1u;
        Waiter wt;
        while (!mbar_test(&sm.empty[slot], par)) {
          if ((*reinterpret_cast<volatile int*>(&sm.abort) || wt.expired(A, flag, t0, SITE_EMPTY))) {
            good = false;
            break;
          }
        }
      }
      if (good) mbar_arrive_expect_tx(&sm.full[slot], static_cast<uint32_t>(cnt) * rb);
    }
    if (!__shfl_sync(0xffffffffu, good ? 1 : 0, 0)) {
      ok = false;
      return;
    }
    if (pitch == rb) {  // unpadded: the stage's rows are one contiguous copy
      if (lane == 0) bulk_g2s(sm.stage[slot], src, static_cast<uint32_t>(cnt) * rb, &sm.full[slot], pol);
    } else {
      for (int r = lane; r < cnt; r += 32)
        bulk_g2s(sm.stage[slot] + static_cast<size_t>(r) * pitch, src + static_cast<size_t>(r) * rb, rb,
                 &sm.full[slot], pol);
    }
    if (lane == 0) stage_stamp<TR>(A, cta, 0, seq);
    ++seq;
  };
  // This CTA's units of a phase: n units split evenly in blocks of `blk`
  // (the gate/up phase splits whole act words: 2 pairs = 4 rows).
  // `pad`: rows at the padded pitch (tensor-core phases) or packed (the logits).
  auto stream = [&](const uint8_t* base, int n, int unit_bytes, int per_stage, int blk, bool pad) {
    const int a = blk * split_begin(cta, n / blk, G), b = blk * split_begin(cta + 1, n / blk, G);
    for (int u = a; u < b && ok; u += per_stage) {
      const int cnt = min(per_stage, b - u);
      issue(base + static_cast<size_t>(u) * unit_bytes, cnt, static_cast<uint32_t>(unit_bytes),
            static_cast<uint32_t>(unit_bytes + (pad ? kRowPad : 0)));
    }
  };
  for (int step = 0; step < nsteps && ok; ++step) {  // the weight sequence repeats every step
      for (int l = 0; l < A.n_layers && ok; ++l) {
        const uint8_t* lw = A.wbase + static_cast<size_t>(l) * A.layer_stride;
        stream(lw + A.off_qkv, S::QKV, S::ROWB_D, S::RPS_D, 1, true);
        stream(lw + A.off_o, S::D, S::ROWB_D, S::RPS_D, 1, true);
        stream(lw + A.off_gu, 2 * S::DFF, S::ROWB_D, S::RPS_D, 4, true);
        stream(lw + A.off_down, S::D, S::ROWB_F, S::RPS_F, 1, true);
      }
      if (ok) stream(A.wbase + A.off_emb, A.vocab, S::ROWB_D, S::RPS_D, 1, false);
    }
    if (lane == 0) {
      // Never leave with copies in flight: wait (bounded) for the last stages
      // issued.  On the normal path they land before the consumers finish.
      const uint32_t first = seq > kStages ? seq - kStages : 0;
      const uint64_t td = globaltimer_ns();
      for (uint32_t s = first; s < seq; ++s) {
        while (!mbar_test(&sm.full[s % kStages], (s / kStages) & 1u)) {
          if (globaltimer_ns() - td > A.wait_ns) break;
        }
      }
    }
  }

  // One attention unit: head h, KV positions [p0, p1) (reference :182-221).
  // Writes o (unnormalised), m, l as exchange words.
  //
  // Layout for latency: a warp owns 16 positions per pass, two lanes per
  // position (each lane holds half of the 64 dims), so QK needs one shuffle per
  // position instead of a full warp reduction; PV is lane-per-dim over
  // probabilities staged in shared memory.  The K/V of the unit's first pass
  // are requested at the start of the layer (att_prefetch), so their latency
  // hides behind the QKV phase.
  struct AttPre {
    uint32_t vbytes;  // bytes of each of the pass's K and V copies in flight (0 = none)
    float rc, rs;     // RoPE cos/sin (threads < 64)
    int unit;         // unit the prefetch belongs to (-1 = none)
  };

  // Issue one pass (up to 128 positions from `base`) of unit (h, j): the cached
  // K and V rows into shared memory by two bulk copies (each contiguous in the
  // cache).  Position `pos` is new: it comes from q/k/v.
  template <class S>
  __device__ __forceinline__ void att_load_pass(const DecodeArgs& A, Smem<S>& sm, AttPre& pre, int l, int pos,
                                                int h, int j, int base) {
    const int t = threadIdx.x;
    const int g = h / S::GQA;
    const int p1 = min(j * A.att_T + A.att_T, pos + 1);
    const size_t half = static_cast<size_t>(S::NKV) * A.ctx * S::DH;
    const __nv_bfloat16* Kc = A.kv + static_cast<size_t>(l) * 2 * half + static_cast<size_t>(g) * A.ctx * S::DH;
    const __nv_bfloat16* Vc = Kc + half;
    const int ncached = max(0, min(min(base + 128, p1), pos) - base);
    pre.vbytes = static_cast<uint32_t>(ncached) * S::DH * 2;
    if (t == 0 && pre.vbytes) {
      const uint64_t pol = l2_policy_evict_last();
      mbar_arrive_expect_tx(&sm.att_bar, 2 * pre.vbytes);
      bulk_g2s(sm.katt, Kc + static_cast<size_t>(base) * S::DH, pre.vbytes, &sm.att_bar, pol);
      bulk_g2s(sm.vatt, Vc + static_cast<size_t>(base) * S::DH, pre.vbytes, &sm.att_bar, pol);
    }
  }

  template <class S>
  __device__ __forceinline__ void att_prefetch(const DecodeArgs& A, Smem<S>& sm, AttPre& pre, int l, int pos,
                                               int u, int nsplit) {
    const int t = threadIdx.x;
    pre.unit = u;
    att_load_pass<S>(A, sm, pre, l, pos, u / nsplit, u % nsplit, (u % nsplit) * A.att_T);
    pre.rc = pre.rs = 0.f;
    if (t < 64) {
      pre.rc = __ldg(A.rcos + static_cast<size_t>(pos) * 32 + (t & 31));
      pre.rs = __ldg(A.rsin + static_cast<size_t>(pos) * 32 + (t & 31));
    }
  }

  template <class S, bool TR>
  __device__ __forceinline__ bool attention_unit(const DecodeArgs& A, Smem<S>& sm, uint32_t flag,
                                                 uint64_t t0, int l, int pos, int u, int nsplit,
                                                 int trace_slot, uint32_t& att_phase, AttPre& pre) {
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int h = u / nsplit, j = u % nsplit;
    const int g = h / S::GQA;
    const int p0 = j * A.att_T, p1 = min(p0 + A.att_T, pos + 1);
    const size_t half = static_cast<size_t>(S::NKV) * A.ctx * S::DH;
    const __nv_bfloat16* Kc = A.kv + static_cast<size_t>(l) * 2 * half + static_cast<size_t>(g) * A.ctx * S::DH;
    const __nv_bfloat16* Vc = Kc + half;
    uint64_t* lw = A.words + static_cast<size_t>(l) * A.layer_words;
    const int qi = lane & 15, hf = lane >> 4;  // position within the warp's 16, dim half

    if (pre.unit != u) att_prefetch<S>(A, sm, pre, l, pos, u, nsplit);
    pre.unit = -1;
    uint32_t& vbytes = pre.vbytes;
    const float rc = pre.rc, rs = pre.rs;
    auto load_pass = [&](int base) { att_load_pass<S>(A, sm, pre, l, pos, h, j, base); };
    // Wait (bounded, ignoring the abort marker) for this pass's V copy; used on
    // every path so the CTA never leaves with the copy in flight.
    auto wait_v = [&]() -> bool {
      if (!vbytes) return true;
      const uint64_t ts0 = globaltimer_ns();
      bool landed = false;
      uint32_t n = 0;
      while (!(landed = mbar_test(&sm.att_bar, att_phase & 1u))) {
        if ((++n & 63u) == 0 && globaltimer_ns() - ts0 > 10000000ull) {
          raise_error(A.ctl, ST_TIMEOUT | SITE_VATT, flag);
          break;
        }
      }
      ++att_phase;
      vbytes = 0;
      return landed;
    };
    // q head h, k/v of kv head g: 3 x 32 word pairs.
    bool ok = gather_pairs<1>(
        A, flag, t0, SITE_QKV,
        [&](int) {
          const int seg = t >> 5, e = (t & 31) * 2;
          const int row = seg == 0 ? h * 64 : (seg == 1 ? S::NH * 64 + g * 64 : (S::NH + S::NKV) * 64 + g * 64);
          return lw + S::D + row + e;
        },
        [&](int) { return t < 96; },
        [&](int, float a, float b) { sm.qkv[2 * t] = a; sm.qkv[2 * t + 1] = b; });
    ok = consumer_sync_and<kConsumers>(ok);
    if (!ok) {
      wait_v();
      return false;
    }
    trace_stamp<TR>(A, trace_slot);
    // RoPE (rotate-half, reference :154-173; f32 tables as model.py:101-107).
    if (t < 64) {
      const int i = t & 31;
      const float* src = sm.qkv + (t < 32 ? 0 : 64);
      const float lo = src[i], hi = src[i + 32];
      float* dst = t < 32 ? sm.rq : sm.rk;
      const float sc = t < 32 ? 0.125f : 1.0f;  // 1/sqrt(64) folded into q (exact)
      dst[i] = (lo * rc - hi * rs) * sc;
      dst[i + 32] = (lo * rs + hi * rc) * sc;
    }
    consumer_sync<kConsumers>();
    const float4* q4 = reinterpret_cast<const float4*>(sm.rq + hf * 32);
    const float vn0 = sm.qkv[128 + 2 * lane], vn1 = sm.qkv[128 + 2 * lane + 1];

    float m = -INFINITY, lsum = 0.f, o0 = 0.f, o1 = 0.f;
    for (int base = p0; base < p1; base += 16 * kConsumerWarps) {
      if (base != p0) load_pass(base);
      if (!__all_sync(0xffffffffu, wait_v())) ok = false;  // K/V rows of this pass landed
      const int pk = base + warp * 16 + qi;
      float sdot = 0.f;
      if (pk == pos) {
  #pragma unroll
        for (int d = 0; d < 32; ++d) sdot = fmaf(sm.rq[hf * 32 + d], sm.rk[hf * 32 + d], sdot);
      } else if (ok && pk < p1) {
        // lane qi starts at chunk qi & 3 so a quarter-warp's 8 rows spread over banks
        const uint4* kr = reinterpret_cast<const uint4*>(sm.katt[pk - base]) + hf * 4;
  #pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int cc = (c + qi) & 3;
          const uint4 kw = kr[cc];
          const float4 qa = q4[2 * cc], qb = q4[2 * cc + 1];
          sdot = fmaf(qa.x, bf16_lo(kw.x), sdot);
          sdot = fmaf(qa.y, bf16_hi(kw.x), sdot);
          sdot = fmaf(qa.z, bf16_lo(kw.y), sdot);
          sdot = fmaf(qa.w, bf16_hi(kw.y), sdot);
          sdot = fmaf(qb.x, bf16_lo(kw.z), sdot);
          sdot = fmaf(qb.y, bf16_hi(kw.z), sdot);
          sdot = fmaf(qb.z, bf16_lo(kw.w), sdot);
          sdot = fmaf(qb.w, bf16_hi(kw.w), sdot);
        }
      }
      sdot += __shfl_xor_sync(0xffffffffu, sdot, 16);
      const bool valid = pk < p1;
      float s = valid ? sdot : -INFINITY;
      float mx = s;
  #pragma unroll
      for (int o = 8; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
      const float mn = fmaxf(m, mx);
      const float pe = valid ? __expf(s - mn) : 0.f;
      float ps = pe;
  #pragma unroll
      for (int o = 8; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
      const float alpha = m == -INFINITY ? 0.f : __expf(m - mn);
      if (hf == 0) sm.wo[warp][qi] = pe;   // stage probabilities for PV
      __syncwarp();
      float a0 = 0.f, a1 = 0.f;
      if (ok) {
  #pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int pv = base + warp * 16 + i;
          const float pi = sm.wo[warp][i];
          float v0 = 0.f, v1 = 0.f;
          if (pv == pos) {
            v0 = vn0; v1 = vn1;
          } else if (pv < p1) {
            const uint32_t vw = reinterpret_cast<const uint32_t*>(sm.vatt[pv - base])[lane];
            v0 = bf16_lo(vw); v1 = bf16_hi(vw);
          }
          a0 = fmaf(pi, v0, a0);
          a1 = fmaf(pi, v1, a1);
        }
      }
      __syncwarp();
      lsum = fmaf(lsum, alpha, ps);
      o0 = fmaf(o0, alpha, a0);
      o1 = fmaf(o1, alpha, a1);
      m = mn;
      // every warp is done reading the staged V before the next pass reuses it
      ok = consumer_sync_and<kConsumers>(ok);
      if (!ok) return false;
    }
    // per-warp state -> shared, then warp 0 merges in fixed order
    sm.wo[warp][2 * lane] = o0;
    sm.wo[warp][2 * lane + 1] = o1;
    if (lane == 0) { sm.wm[warp] = m; sm.wl[warp] = lsum; }
    consumer_sync<kConsumers>();
    if (warp == 0) {
      float M = -INFINITY;
  #pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.wm[w]);
      float L = 0.f, b0 = 0.f, b1 = 0.f;
  #pragma unroll
      for (int w = 0; w < kConsumerWarps; ++w) {
        const float e = sm.wl[w] > 0.f ? __expf(sm.wm[w] - M) : 0.f;
        L = fmaf(sm.wl[w], e, L);
        b0 = fmaf(sm.wo[w][2 * lane], e, b0);
        b1 = fmaf(sm.wo[w][2 * lane + 1], e, b1);
      }
      uint64_t* out = lw + A.w_att + static_cast<size_t>(h * nsplit + j) * kAttWords;
      st_word(out + 2 * lane, b0, flag);
      st_word(out + 2 * lane + 1, b1, flag);
      if (lane == 0) {
        st_word(out + 64, M, flag);
        st_word(out + 65, L, flag);
      }
    }
    // The first head of the group, owning the split that holds `pos`, appends
    // this position's K (post-RoPE) and V to the cache in bf16.
    if (warp == 1 && (h % S::GQA) == 0 && pos >= p0 && pos < p1) {
      __nv_bfloat162 kk = __floats2bfloat162_rn(sm.rk[2 * lane], sm.rk[2 * lane + 1]);
      __nv_bfloat162 vv = __floats2bfloat162_rn(vn0, vn1);
      __nv_bfloat16* kd = const_cast<__nv_bfloat16*>(Kc) + static_cast<size_t>(pos) * S::DH;
      __nv_bfloat16* vd = const_cast<__nv_bfloat16*>(Vc) + static_cast<size_t>(pos) * S::DH;
      reinterpret_cast<__nv_bfloat162*>(kd)[lane] = kk;
      reinterpret_cast<__nv_bfloat162*>(vd)[lane] = vv;
    }
    consumer_sync<kConsumers>();
    return true;
  }

  template <class S, bool TR>
  __global__ void __launch_bounds__(kThreads, 1) decode_b1_kernel(const DecodeArgs A) {
    extern __shared__ __align__(128) uint8_t decode_smem_raw[];
    static_assert(SmemChecks<S>::ok, "");
    Smem<S>& sm = *reinterpret_cast<Smem<S>*>(decode_smem_raw);
    const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
    const int cta = blockIdx.x;
    const int G = A.grid_part;
    const uint64_t t0 = globaltimer_ns();

    // A workspace holding an earlier device error stays halted until reset.
    if (ld_relaxed_u32(&A.ctl->status) != 0u) return;
    const int nsteps = A.n_steps > 1 ? A.n_steps : 1;
    const int tok0 = A.tok ? __ldg(A.tok) : A.tok_val, pos0 = A.pos ? __ldg(A.pos) : A.pos_val;
    if (tok0 < 0 || tok0 >= A.vocab || pos0 < 0 || pos0 + nsteps > A.ctx) {
      if (cta == 0 && t == 0)
        atomicCAS(&A.ctl->status, 0u, ST_BAD_INPUT | (tok0 < 0 || tok0 >= A.vocab ? 1u : 2u));
      return;
    }
    // Step s writes its exchange words with flag0 + s; gen holds the last flag used.
    const uint32_t flag0 = ld_relaxed_u32(&A.ctl->gen) + 1u;

    if (t == 0) {
      for (int s = 0; s < kStages; ++s) {
        mbar_init(&sm.full[s], 1);
        mbar_init(&sm.empty[s], kConsumerWarps);
      }
      mbar_init(&sm.att_bar, 1);
      sm.abort = 0;
      fence_mbar_init();
    }
    if (t < kPhases) {  // each phase's unit range for this CTA (the producer streams the same ranges)
      const int n = t == PH_QKV ? S::QKV : t == PH_GU ? S::DFF / 2 : t == PH_VOCAB ? A.vocab : S::D;
      const int blk = t == PH_GU ? 4 : 1;  // gate/up: whole act words of 4 rows
      sm.rng[2 * t] = blk * split_begin(cta, n, G);
      sm.rng[2 * t + 1] = blk * split_begin(cta + 1, n, G);
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
      producer_loop<S, TR>(A, sm, cta, flag0, t0, nsteps);  // the whole producer warp
      return;
    }

    Ring ring{sm.stage, sm.full, sm.empty, 0u};
    bool ok = true;
    uint32_t att_phase = 0;  // completed uses of sm.att_bar
    AttPre pre;
    pre.unit = -1;
    pre.vbytes = 0;
    trace_stamp<TR>(A, 0);
    const int tf = 1 + A.n_layers * kTracePerLayer;
    for (int step = 0; step < nsteps && ok; ++step) {
    const uint32_t flag = flag0 + static_cast<uint32_t>(step);
    const int pos = pos0 + step;
    int tok = tok0;
    if (step > 0) {  // the previous step's argmax, published by the CTA that finished it
      if (t == 0) {
        Waiter wt;
        uint64_t w = ld_acquire_u64(&A.ctl->tok_word);
        while (static_cast<uint32_t>(w >> 32) != flag - 1u) {
          if (wt.expired(A, flag, t0, SITE_TOKEN)) {
            ok = false;
            break;
          }
          w = ld_acquire_u64(&A.ctl->tok_word);
        }
        sm.tok_in = static_cast<int>(static_cast<uint32_t>(w));
      }
      ok = consumer_sync_and<kConsumers>(ok);
      if (!ok) break;
      // K/V rows the previous step appended (other CTAs, generic stores) are read
      // below by bulk copies (async proxy)
      fence_proxy_async_all();
      tok = sm.tok_in;
    }
    const int nsplit = (pos + A.att_T) / A.att_T;  // ceil((pos+1)/T)
    const int n_units = S::NH * nsplit;

    for (int l = 0; l < A.n_layers; ++l) {
      uint64_t* lw = A.words + static_cast<size_t>(l) * A.layer_words;
      if (cta < n_units) att_prefetch<S>(A, sm, pre, l, pos, cta, nsplit);  // K/V of this layer's unit
      // ---- residual in: the embedding row (reference :87-88) or H_l, written
      // by layer l-1's down phase; RMSNorm1 -> x ----
      if (l == 0) {
        constexpr int NP = S::NP_D;
        float2 g[NP];
        load_gain_pairs<S, NP>(A.ln1, g);
        const uint32_t* e = reinterpret_cast<const uint32_t*>(A.wbase + A.off_emb) +
                            static_cast<size_t>(tok) * (S::D / 2);
        float hv[NP][2];
#pragma unroll
        for (int i = 0; i < NP; ++i) {
          const int k = t + i * kConsumers;
          const uint32_t w2 = k < S::D / 2 ? __ldg(e + k) : 0u;
          hv[i][0] = bf16_lo(w2);
          hv[i][1] = bf16_hi(w2);
        }
        ok = norm_pairs<S, NP>(sm, hv, g, A.eps, true);
      } else {
        ok = gather_norm<S>(A, sm, lw, flag, t0, SITE_H, A.ln1 + static_cast<size_t>(l) * S::D);
      }
      if (!ok) break;
      const int ts = 1 + l * kTracePerLayer;
      trace_stamp<TR>(A, ts + 0);
      trace_stamp<TR>(A, ts + 1);
      // ---- QKV rows -> exchange words ----
      {
        ok = gemv_phase<S::D, S::PITCH_D, S::RPS_D, S::MT_QKV, 16 * S::MT_MAX, TR>(
            A, ring, &sm.part[0][0], sm.xb, flag, t0, sm.rng[2 * PH_QKV], sm.rng[2 * PH_QKV + 1],
            [&](int u, float v) { st_word(lw + S::D + u, v, flag); });
        if (!ok) break;
      }
      trace_stamp<TR>(A, ts + 2);
      trace_stamp<TR>(A, ts + 3);  // rewritten by a CTA that runs an attention unit
      // ---- attention units ----
      for (int u = cta; u < n_units && ok; u += G) {
        ok = attention_unit<S, TR>(A, sm, flag, t0, l, pos, u, nsplit, ts + 3, att_phase, pre);
      }
      if (!ok) break;
      trace_stamp<TR>(A, ts + 4);
      // ---- gather attention partials, merge splits -> x (bf16) ----
      // Item 0 (threads < NH*nsplit): the (m, l) pair of unit t -> shared memory.
      // Items 1..2*nsplit: this thread's 4 output dims of head t/16 per split.
      {
        float va[2 * kMaxSplits], vb[2 * kMaxSplits];
        const int hh = t >> 4, d0 = (t & 15) * 4;
        ok = gather_pairs<1 + 2 * kMaxSplits, 3>(  // groups of 3: (m, l) + one split's 4 dims
            A, flag, t0, SITE_ATT,
            [&](int i) {
              if (i == 0) return lw + A.w_att + static_cast<size_t>(t) * kAttWords + 64;
              const int jj = (i - 1) >> 1, r = (i - 1) & 1;
              return lw + A.w_att + static_cast<size_t>(hh * nsplit + jj) * kAttWords + d0 + 2 * r;
            },
            [&](int i) { return i == 0 ? t < n_units : (hh < S::NH && ((i - 1) >> 1) < nsplit); },
            [&](int i, float a, float b) {
              if (i == 0) { sm.ml[2 * t] = a; sm.ml[2 * t + 1] = b; }
              else { va[i - 1] = a; vb[i - 1] = b; }
            });
        ok = consumer_sync_and<kConsumers>(ok);
        if (!ok) break;
        trace_stamp<TR>(A, ts + 5);
        if (hh < S::NH) {
          const float* ml = sm.ml + 2 * hh * nsplit;
          float M = -INFINITY;
          for (int jj = 0; jj < nsplit; ++jj) M = fmaxf(M, ml[2 * jj]);
          float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
  #pragma unroll
          for (int jj = 0; jj < kMaxSplits; ++jj) {
            if (jj < nsplit) {
              const float e = __expf(ml[2 * jj] - M);
              L = fmaf(ml[2 * jj + 1], e, L);
              o[0] = fmaf(va[2 * jj], e, o[0]);
              o[1] = fmaf(vb[2 * jj], e, o[1]);
              o[2] = fmaf(va[2 * jj + 1], e, o[2]);
              o[3] = fmaf(vb[2 * jj + 1], e, o[3]);
            }
          }
          const float inv = 1.0f / fmaxf(L, 1e-10f);
          __nv_bfloat162* xo = reinterpret_cast<__nv_bfloat162*>(sm.xb) + (hh * 64 + d0) / 2;
          xo[0] = __floats2bfloat162_rn(o[0] * inv, o[1] * inv);
          xo[1] = __floats2bfloat162_rn(o[2] * inv, o[3] * inv);
        }
        consumer_sync<kConsumers>();
      }
      trace_stamp<TR>(A, ts + 6);
      // ---- O rows: HM = H + attn @ Wo^T ----
      {
        ok = gemv_phase<S::D, S::PITCH_D, S::RPS_D, S::MT_O, 16 * S::MT_MAX, TR>(
            A, ring, &sm.part[0][0], sm.xb, flag, t0, sm.rng[2 * PH_O], sm.rng[2 * PH_O + 1],
            [&](int u, float v) { st_word(lw + A.w_hm + u, sm.h[u] + v, flag); });
        if (!ok) break;
      }
      trace_stamp<TR>(A, ts + 7);
      // ---- gather HM (the residual after attention); RMSNorm2 -> x ----
      ok = gather_norm<S>(A, sm, lw + A.w_hm, flag, t0, SITE_HM, A.ln2 + static_cast<size_t>(l) * S::D);
      if (!ok) break;
      trace_stamp<TR>(A, ts + 8);
      trace_stamp<TR>(A, ts + 9);
      // ---- gate/up rows -> act = silu(g) * u; an exchange word holds two acts ----
      {
        const int a = sm.rng[2 * PH_GU], b = sm.rng[2 * PH_GU + 1];
        ok = gemv_phase<S::D, S::PITCH_D, S::RPS_D, S::MT_GU, 16 * S::MT_MAX, TR>(
            A, ring, &sm.part[0][0], sm.xb, flag, t0, a, b, [&](int u, float v) { sm.gu_out[u - a] = v; });
        if (!ok) break;
        consumer_sync<kConsumers>();  // gu_out complete
        // rows 4i .. 4i + 3 of the CTA's range: gate, up of pair 2m, gate, up of pair 2m + 1
        if (t < (b - a) / 4) {
          const float4 gu = reinterpret_cast<const float4*>(sm.gu_out)[t];
          const float a0 = gu.x * (1.0f / (1.0f + __expf(-gu.x))) * gu.y;
          const float a1 = gu.z * (1.0f / (1.0f + __expf(-gu.z))) * gu.w;
          const __nv_bfloat162 pk = __floats2bfloat162_rn(a0, a1);
          st_word(lw + A.w_act + a / 4 + t, __uint_as_float(*reinterpret_cast<const uint32_t*>(&pk)), flag);
        }
      }
      trace_stamp<TR>(A, ts + 10);
      // ---- gather act -> x (bf16), down rows: H_{l+1} = HM + act @ Wd^T ----
      {
        // word m holds act[2m] (low half) and act[2m + 1]; thread t reads word
        // pairs p = t + 256 i, i.e. act[4p .. 4p + 3]
        ok = gather_pairs<S::NP_ACT>(
            A, flag, t0, SITE_ACT, [&](int i) { return lw + A.w_act + 2 * (t + i * kConsumers); },
            [&](int i) { return t + i * kConsumers < S::DFF / 4; },
            [&](int i, float a, float b) {  // the payloads are the bf16 pairs, in order
              reinterpret_cast<uint2*>(sm.xb)[t + i * kConsumers] = make_uint2(__float_as_uint(a), __float_as_uint(b));
            });
        ok = consumer_sync_and<kConsumers>(ok);
        if (!ok) break;
        trace_stamp<TR>(A, ts + 11);
        uint64_t* nxt = A.words + static_cast<size_t>(l + 1) * A.layer_words;  // H_{l+1} at word 0
        ok = gemv_phase<S::DFF, S::PITCH_F, S::RPS_F, S::MT_DOWN, 16 * S::MT_MAX, TR>(
            A, ring, &sm.part[0][0], sm.xb, flag, t0, sm.rng[2 * PH_DOWN], sm.rng[2 * PH_DOWN + 1],
            [&](int u, float v) { st_word(nxt + u, sm.h[u] + v, flag); });
        if (!ok) break;
      }
      trace_stamp<TR>(A, ts + 12);
    }

    if (ok) {
      // ---- final norm + tied logits + argmax (reference :314-357) ----
      uint64_t* fw = A.words + static_cast<size_t>(A.n_layers) * A.layer_words;
      ok = gather_norm<S>(A, sm, fw, flag, t0, SITE_FINAL, A.lnf);
    }
    trace_stamp<TR>(A, tf + 0);
    if (ok) {
      const XSmem x{reinterpret_cast<const uint4*>(sm.xb)};
      float best_v = -INFINITY;
      int best_i = 0x7fffffff;
      ok = gemv_phase_wide<S::KD, S::ROWB_D, S::RPS_D>(A, ring, flag, t0, sm.rng[2 * PH_VOCAB],
                                                       sm.rng[2 * PH_VOCAB + 1], x,
                                                       [&](int u, float v, float) {
                                                         if (lane == 0 && A.logits) A.logits[u] = v;
                                                         if (v > best_v) { best_v = v; best_i = u; }
                                                       });
      ok = consumer_sync_and<kConsumers>(ok);
      trace_stamp<TR>(A, tf + 1);
      if (ok) {
        if (lane == 0) { sm.am_v[warp] = best_v; sm.am_i[warp] = best_i; }
        consumer_sync<kConsumers>();
        if (t == 0) {
          float bv = sm.am_v[0];
          int bi = sm.am_i[0];
          for (int w = 1; w < kConsumerWarps; ++w) {
            if (sm.am_v[w] > bv || (sm.am_v[w] == bv && sm.am_i[w] < bi)) { bv = sm.am_v[w]; bi = sm.am_i[w]; }
          }
          A.am_val[cta] = bv;
          A.am_idx[cta] = bi;
          __threadfence();
          const uint32_t ticket = atomicAdd(&A.ctl->arrive, 1u);
          if (ticket == static_cast<uint32_t>(gridDim.x) - 1u) {
            __threadfence();
            float gv = -INFINITY;
            int gi = 0x7fffffff;
            for (int c = 0; c < static_cast<int>(gridDim.x); ++c) {
              const float v = *reinterpret_cast<volatile float*>(&A.am_val[c]);
              const int i = *reinterpret_cast<volatile int*>(&A.am_idx[c]);
              if (v > gv || (v == gv && i < gi)) { gv = v; gi = i; }
            }
            const int tk = gi == 0x7fffffff ? 0 : gi;
            *A.next_tok = tk;
            if (A.tok_out != nullptr) A.tok_out[step] = tk;
            A.ctl->arrive = 0u;
            __threadfence();
            st_relaxed_u32(&A.ctl->gen, flag);
            if (step + 1 < nsteps)  // the next step's input
              st_release_u64(&A.ctl->tok_word, (static_cast<uint64_t>(flag) << 32) | static_cast<uint32_t>(tk));
          }
        }
      }
    }
  }  // step
  trace_stamp<TR>(A, tf + 2);
  if (!ok) {
    // a K/V staging copy requested for an attention unit that never ran
    if (pre.vbytes) {
      const uint64_t ts0 = globaltimer_ns();
      while (!mbar_test(&sm.att_bar, att_phase & 1u) && globaltimer_ns() - ts0 < 10000000ull) {
      }
    }
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
  }
}

}  // namespace b2d
