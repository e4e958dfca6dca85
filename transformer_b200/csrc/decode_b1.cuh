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

#include "b2d_ptx.cuh"

namespace b2d {

// Device status word (Control::status).  0 = ok.
enum : uint32_t {
  ST_TIMEOUT = 0x100u,    // | site
  ST_BAD_INPUT = 0x200u,  // | 1 token, 2 pos
};
enum : uint32_t {
  SITE_H = 1, SITE_QKV = 2, SITE_ATT = 3, SITE_HM = 4, SITE_ACT = 5, SITE_FINAL = 6,
  SITE_FULL = 7, SITE_EMPTY = 8, SITE_DRAIN = 9,
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
};

struct DecodeArgs {
  const uint8_t* wbase;  // packed weights (see include/b2d.h layout)
  uint64_t layer_stride, off_qkv, off_o, off_gu, off_down, off_emb;
  const float* ln1;  // [L][D]
  const float* ln2;  // [L][D]
  const float* lnf;  // [D]
  const float* rcos; // [ctx][DH/2]
  const float* rsin;
  const int32_t* tok;
  const int32_t* pos;
  __nv_bfloat16* kv;  // [L][2][NKV][ctx][DH]
  float* logits;      // [V] or null
  int32_t* next_tok;
  uint64_t* words;    // exchange words
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
};

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kThreads = kConsumers + 32;
constexpr int kStageBytes = 16896;  // 8 rows x 2 KB or 3 rows x 5.5 KB (306M shapes)
constexpr int kStages = 12;
constexpr int kAttWords = 66;       // per attention unit: o[64], m, l
constexpr int kMaxSplits = 8;       // attention units per head

template <int D_, int DFF_, int NH_, int NKV_>
struct Shape {
  static constexpr int D = D_, DFF = DFF_, NH = NH_, NKV = NKV_, DH = 64;
  static constexpr int GQA = NH / NKV;
  static constexpr int QKV = (NH + 2 * NKV) * DH;
  static constexpr int KD = D / 256;    // 16-byte chunks per lane along K = D
  static constexpr int KF = DFF / 256;  // along K = DFF
  static constexpr int ROWB_D = 2 * D;
  static constexpr int ROWB_F = 2 * DFF;
  static constexpr int RPS_D = kStageBytes / ROWB_D;        // rows of K=D per stage
  static constexpr int PPS = kStageBytes / (2 * ROWB_D);    // gate/up pairs per stage
  static constexpr int RPS_F = kStageBytes / ROWB_F;        // down rows per stage
  static constexpr int XMAX = DFF > D ? DFF : D;
  static_assert(D % 256 == 0 && DFF % 256 == 0, "row length must be a multiple of 256");
  static_assert(RPS_D >= 1 && PPS >= 1 && RPS_F >= 1, "stage too small");
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
  float x[S::XMAX];       // GEMV input (bf16-rounded values)
  float qkv[3 * 64];      // attention unit inputs
  float rq[64], rk[64];   // post-RoPE q (pre-scaled), k
  float wm[kConsumerWarps], wl[kConsumerWarps];
  float wo[kConsumerWarps][64];
  float red[kConsumerWarps];
  float ml[2 * kConsumers];  // (m, l) of each attention unit
  float am_v[kConsumerWarps];
  int am_i[kConsumerWarps];
  int abort;
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

// Gather up to N word pairs per thread.  addr(i) -> pointer to pair i (16-B
// aligned); valid(i) says whether this thread owns item i; store(i, a, b)
// receives the payloads.  All owned loads are issued together, then the
// thread spins on one pending pair at a time.  Returns false on timeout/abort.
template <int N, class AddrF, class ValidF, class StoreF>
__device__ __forceinline__ bool gather_pairs(const DecodeArgs& A, uint32_t flag, uint64_t t0,
                                             uint32_t site, AddrF addr, ValidF valid, StoreF store) {
  static_assert(N <= 32, "pending mask is 32 bits");
  constexpr int GRP = 8;  // loads issued together per thread
  uint32_t pending = 0;
#pragma unroll
  for (int i = 0; i < N; ++i)
    if (valid(i)) pending |= 1u << i;
  uint32_t spins = 0;
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
      if ((++spins & 31u) == 0 && wait_expired(A, flag, t0, site)) return false;
    }
  }
  return true;
}

// Consumer-side view of the stage ring.
struct Ring {
  uint8_t (*stage)[kStageBytes];
  uint64_t* full;
  uint64_t* empty;
  uint32_t seq;
};

// Warp-uniform: every lane acquires the stage itself; lane 0 decides timeouts.
__device__ __forceinline__ bool wait_full(const DecodeArgs& A, Ring& r, uint32_t flag, uint64_t t0) {
  const uint32_t slot = r.seq % kStages, par = (r.seq / kStages) & 1u;
  const int lane = threadIdx.x & 31;
  uint32_t spins = 0;
  while (true) {
    const bool done = mbar_test(&r.full[slot], par);
    if (__all_sync(0xffffffffu, done)) return true;
    if ((++spins & 63u) == 0) {
      const bool exp = lane == 0 ? wait_expired(A, flag, t0, SITE_FULL) : false;
      if (__shfl_sync(0xffffffffu, exp ? 1 : 0, 0)) return false;
    }
  }
}

// One GEMV phase over this CTA's units [u_begin, u_end) (a unit is one row, or
// a gate/up row pair when PAIR), streamed in stages of `per_stage` units.
// Warp w takes units u with (u - u_begin) % 8 == w.  out(u, dot0, dot1) is
// called on every lane with the warp-reduced dot products.
template <int KI, int ROWB, bool PAIR, class Out>
__device__ __forceinline__ bool gemv_phase(const DecodeArgs& A, Ring& ring, uint32_t flag, uint64_t t0,
                                           int u_begin, int u_end, int per_stage,
                                           const uint4 (&x)[KI], Out out) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int UNIT_BYTES = PAIR ? 2 * ROWB : ROWB;
  bool ok = true;
  for (int u0 = u_begin; u0 < u_end; u0 += per_stage) {
    const int u1 = min(u0 + per_stage, u_end);
    if (ok) ok = wait_full(A, ring, flag, t0);
    const uint32_t slot = ring.seq % kStages;
    if (ok) {
      const uint8_t* sb = ring.stage[slot];
      const int first = u0 + ((warp - (u0 - u_begin)) % kConsumerWarps + kConsumerWarps) % kConsumerWarps;
      for (int u = first; u < u1; u += kConsumerWarps) {
        const uint4* rp = reinterpret_cast<const uint4*>(sb + static_cast<size_t>(u - u0) * UNIT_BYTES);
        float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
        for (int k = 0; k < KI; ++k) acc0 = dot8(rp[k * 32 + lane], x[k], acc0);
        if (PAIR) {
          const uint4* rq = rp + ROWB / 16;
#pragma unroll
          for (int k = 0; k < KI; ++k) acc1 = dot8(rq[k * 32 + lane], x[k], acc1);
        }
        acc0 = warp_sum(acc0);
        if (PAIR) acc1 = warp_sum(acc1);
        out(u, acc0, acc1);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&ring.empty[slot]);
    ring.seq++;
    if (!ok) return false;
  }
  return true;
}

// Lane l holds x[k*256 + l*8 .. +8) as packed bf16 pairs (matches the
// weight chunk it reads from the stage).
template <class S, int KI>
__device__ __forceinline__ void load_x(const float* xs, uint4 (&x)[KI]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < KI; ++k) {
    const float4* p = reinterpret_cast<const float4*>(xs + k * 256 + lane * 8);
    const float4 a = p[0], b = p[1];
    x[k] = make_uint4(pack_bf16x2(a.x, a.y), pack_bf16x2(a.z, a.w), pack_bf16x2(b.x, b.y),
                      pack_bf16x2(b.z, b.w));
  }
}

// x = bf16(h * rsqrt(mean(h^2) + eps) * g)  (RMSNorm, reference :121-126)
template <class S>
__device__ __forceinline__ void rmsnorm_to_x(Smem<S>& sm, const float* g, float eps) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  float ss = 0.f;
#pragma unroll
  for (int i = t; i < S::D; i += kConsumers) ss = fmaf(sm.h[i], sm.h[i], ss);
  ss = warp_sum(ss);
  if (lane == 0) sm.red[warp] = ss;
  consumer_sync<kConsumers>();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) tot += sm.red[w];
  const float r = rsqrtf(tot / static_cast<float>(S::D) + eps);
  for (int i = t; i < S::D; i += kConsumers) sm.x[i] = round_bf16(sm.h[i] * r * __ldg(g + i));
  consumer_sync<kConsumers>();
}

// Producer: streams this CTA's weight ranges for the whole step.
template <class S>
__device__ void producer_loop(const DecodeArgs& A, Smem<S>& sm, int cta, uint32_t flag, uint64_t t0) {
  const uint64_t pol = l2_policy_evict_first();
  const int G = A.grid_part;
  uint32_t seq = 0;
  bool ok = true;
  auto issue = [&](const uint8_t* src, uint32_t bytes) {
    const uint32_t slot = seq % kStages;
    if (seq >= kStages) {
      const uint32_t par = ((seq / kStages) - 1) & 1u;
      uint32_t spins = 0;
      while (!mbar_test(&sm.empty[slot], par)) {
        if (((++spins & 63u) == 0) &&
            (*reinterpret_cast<volatile int*>(&sm.abort) || wait_expired(A, flag, t0, SITE_EMPTY))) {
          ok = false;
          return;
        }
      }
    }
    mbar_arrive_expect_tx(&sm.full[slot], bytes);
    bulk_g2s(sm.stage[slot], src, bytes, &sm.full[slot], pol);
    ++seq;
  };
  auto stream = [&](const uint8_t* base, int n, int unit_bytes, int per_stage) {
    const int a = split_begin(cta, n, G), b = split_begin(cta + 1, n, G);
    for (int u = a; u < b && ok; u += per_stage) {
      const int cnt = min(per_stage, b - u);
      issue(base + static_cast<size_t>(u) * unit_bytes, static_cast<uint32_t>(cnt * unit_bytes));
    }
  };
  for (int l = 0; l < A.n_layers && ok; ++l) {
    const uint8_t* lw = A.wbase + static_cast<size_t>(l) * A.layer_stride;
    stream(lw + A.off_qkv, S::QKV, S::ROWB_D, S::RPS_D);
    stream(lw + A.off_o, S::D, S::ROWB_D, S::RPS_D);
    stream(lw + A.off_gu, S::DFF, 2 * S::ROWB_D, S::PPS);
    stream(lw + A.off_down, S::D, S::ROWB_F, S::RPS_F);
  }
  if (ok) stream(A.wbase + A.off_emb, A.vocab, S::ROWB_D, S::RPS_D);
  {
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
template <class S>
__device__ __forceinline__ bool attention_unit(const DecodeArgs& A, Smem<S>& sm, uint32_t flag,
                                               uint64_t t0, int l, int pos, int h, int j, int nsplit) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int g = h / S::GQA;
  const int p0 = j * A.att_T, p1 = min(p0 + A.att_T, pos + 1);
  const size_t half = static_cast<size_t>(S::NKV) * A.ctx * S::DH;
  const __nv_bfloat16* Kc = A.kv + static_cast<size_t>(l) * 2 * half + static_cast<size_t>(g) * A.ctx * S::DH;
  const __nv_bfloat16* Vc = Kc + half;
  uint64_t* lw = A.words + static_cast<size_t>(l) * A.layer_words;

  // Prefetch the first 64 positions' K/V (lane holds dims 2*lane, 2*lane+1)
  // while the q/k/v words are still in flight.
  uint32_t kr[8], vr[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int p = p0 + warp + 8 * i;
    kr[i] = vr[i] = 0u;
    if (p < p1 && p < pos) {
      kr[i] = __ldg(reinterpret_cast<const unsigned int*>(Kc + static_cast<size_t>(p) * S::DH) + lane);
      vr[i] = __ldg(reinterpret_cast<const unsigned int*>(Vc + static_cast<size_t>(p) * S::DH) + lane);
    }
  }
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
  if (!ok) return false;
  // RoPE (rotate-half, reference :154-173; f32 tables as model.py:101-107).
  if (t < 64) {
    const int i = t & 31;
    const float* src = sm.qkv + (t < 32 ? 0 : 64);
    const float c = __ldg(A.rcos + static_cast<size_t>(pos) * 32 + i);
    const float s = __ldg(A.rsin + static_cast<size_t>(pos) * 32 + i);
    const float lo = src[i], hi = src[i + 32];
    float* dst = t < 32 ? sm.rq : sm.rk;
    const float sc = t < 32 ? 0.125f : 1.0f;  // 1/sqrt(64) folded into q (exact)
    dst[i] = (lo * c - hi * s) * sc;
    dst[i + 32] = (lo * s + hi * c) * sc;
  }
  consumer_sync<kConsumers>();
  const float q0 = sm.rq[2 * lane], q1 = sm.rq[2 * lane + 1];
  const float kn0 = sm.rk[2 * lane], kn1 = sm.rk[2 * lane + 1];
  const float vn0 = sm.qkv[128 + 2 * lane], vn1 = sm.qkv[128 + 2 * lane + 1];

  float m = -INFINITY, lsum = 0.f, o0 = 0.f, o1 = 0.f;
  for (int base = p0; base < p1; base += 64) {
    if (base != p0) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int p = base + warp + 8 * i;
        kr[i] = vr[i] = 0u;
        if (p < p1 && p < pos) {
          kr[i] = __ldg(reinterpret_cast<const unsigned int*>(Kc + static_cast<size_t>(p) * S::DH) + lane);
          vr[i] = __ldg(reinterpret_cast<const unsigned int*>(Vc + static_cast<size_t>(p) * S::DH) + lane);
        }
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int p = base + warp + 8 * i;
      if (p < p1) {
        float k0, k1, v0, v1;
        if (p == pos) {
          k0 = kn0; k1 = kn1; v0 = vn0; v1 = vn1;
        } else {
          k0 = bf16_lo(kr[i]); k1 = bf16_hi(kr[i]);
          v0 = bf16_lo(vr[i]); v1 = bf16_hi(vr[i]);
        }
        const float s = warp_sum(fmaf(q0, k0, q1 * k1));
        const float mn = fmaxf(m, s);
        const float alpha = __expf(m - mn);
        const float pe = __expf(s - mn);
        lsum = fmaf(lsum, alpha, pe);
        o0 = fmaf(o0, alpha, pe * v0);
        o1 = fmaf(o1, alpha, pe * v1);
        m = mn;
      }
    }
  }
  sm.wo[warp][2 * lane] = o0;
  sm.wo[warp][2 * lane + 1] = o1;
  if (lane == 0) { sm.wm[warp] = m; sm.wl[warp] = lsum; }
  consumer_sync<kConsumers>();
  if (warp == 0) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.wm[w]);
    float L = 0.f, a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float e = sm.wl[w] > 0.f ? __expf(sm.wm[w] - M) : 0.f;
      L = fmaf(sm.wl[w], e, L);
      a0 = fmaf(sm.wo[w][2 * lane], e, a0);
      a1 = fmaf(sm.wo[w][2 * lane + 1], e, a1);
    }
    uint64_t* out = lw + A.w_att + static_cast<size_t>(h * nsplit + j) * kAttWords;
    st_word(out + 2 * lane, a0, flag);
    st_word(out + 2 * lane + 1, a1, flag);
    if (lane == 0) {
      st_word(out + 64, M, flag);
      st_word(out + 65, L, flag);
    }
  }
  // The first head of the group, owning the split that holds `pos`, appends
  // this position's K (post-RoPE) and V to the cache in bf16.
  if (warp == 1 && (h % S::GQA) == 0 && pos >= p0 && pos < p1) {
    __nv_bfloat162 kk = __floats2bfloat162_rn(kn0, kn1);
    __nv_bfloat162 vv = __floats2bfloat162_rn(vn0, vn1);
    __nv_bfloat16* kd = const_cast<__nv_bfloat16*>(Kc) + static_cast<size_t>(pos) * S::DH;
    __nv_bfloat16* vd = const_cast<__nv_bfloat16*>(Vc) + static_cast<size_t>(pos) * S::DH;
    reinterpret_cast<__nv_bfloat162*>(kd)[lane] = kk;
    reinterpret_cast<__nv_bfloat162*>(vd)[lane] = vv;
  }
  consumer_sync<kConsumers>();
  return true;
}

template <class S>
__global__ void __launch_bounds__(kThreads, 1) decode_b1_kernel(const DecodeArgs A) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem<S>& sm = *reinterpret_cast<Smem<S>*>(smem_raw);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int cta = blockIdx.x;
  const int G = A.grid_part;
  const uint64_t t0 = globaltimer_ns();

  // A workspace holding an earlier device error stays halted until reset.
  if (ld_relaxed_u32(&A.ctl->status) != 0u) return;
  const int tok = __ldg(A.tok), pos = __ldg(A.pos);
  if (tok < 0 || tok >= A.vocab || pos < 0 || pos >= A.ctx) {
    if (cta == 0 && t == 0) atomicCAS(&A.ctl->status, 0u, ST_BAD_INPUT | (tok < 0 || tok >= A.vocab ? 1u : 2u));
    return;
  }
  const uint32_t flag = ld_relaxed_u32(&A.ctl->gen) + 1u;

  if (t == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    sm.abort = 0;
    fence_mbar_init();
  }
  __syncthreads();

  if (warp == kConsumerWarps) {
    if (lane == 0) producer_loop<S>(A, sm, cta, flag, t0);
    return;
  }

  Ring ring{sm.stage, sm.full, sm.empty, 0u};
  bool ok = true;
  const int nsplit = (pos + A.att_T) / A.att_T;  // ceil((pos+1)/T)
  const int n_units = S::NH * nsplit;

  // Embedding row (reference :87-88).
  {
    const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(A.wbase + A.off_emb) +
                             static_cast<size_t>(tok) * S::D;
    for (int i = t; i < S::D; i += kConsumers) sm.h[i] = __bfloat162float(e[i]);
  }
  consumer_sync<kConsumers>();

  uint4 xr[S::KD];
  for (int l = 0; l < A.n_layers; ++l) {
    uint64_t* lw = A.words + static_cast<size_t>(l) * A.layer_words;
    // ---- residual in: H_l (written by layer l-1's down phase) ----
    if (l > 0) {
      ok = gather_pairs<(S::D / 2 + kConsumers - 1) / kConsumers>(
          A, flag, t0, SITE_H, [&](int i) { return lw + 2 * (t + i * kConsumers); },
          [&](int i) { return t + i * kConsumers < S::D / 2; },
          [&](int i, float a, float b) { const int k = t + i * kConsumers; sm.h[2 * k] = a; sm.h[2 * k + 1] = b; });
      ok = consumer_sync_and<kConsumers>(ok);
      if (!ok) break;
    }
    rmsnorm_to_x<S>(sm, A.ln1 + static_cast<size_t>(l) * S::D, A.eps);
    load_x<S, S::KD>(sm.x, xr);
    // ---- QKV rows -> exchange words ----
    {
      const int a = split_begin(cta, S::QKV, G), b = split_begin(cta + 1, S::QKV, G);
      ok = gemv_phase<S::KD, S::ROWB_D, false>(A, ring, flag, t0, a, b, S::RPS_D, xr,
                                               [&](int u, float v, float) {
                                                 if (lane == 0) st_word(lw + S::D + u, v, flag);
                                               });
      ok = consumer_sync_and<kConsumers>(ok);
      if (!ok) break;
    }
    // ---- attention units ----
    for (int u = cta; u < n_units && ok; u += G) {
      ok = attention_unit<S>(A, sm, flag, t0, l, pos, u / nsplit, u % nsplit, nsplit);
    }
    if (!ok) break;
    // ---- gather attention partials, merge splits -> x (bf16) ----
    // Item 0 (threads < NH*nsplit): the (m, l) pair of unit t -> shared memory.
    // Items 1..2*nsplit: this thread's 4 output dims of head t/16 per split.
    {
      float va[2 * kMaxSplits], vb[2 * kMaxSplits];
      const int hh = t >> 4, d0 = (t & 15) * 4;
      ok = gather_pairs<1 + 2 * kMaxSplits>(
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
#pragma unroll
        for (int k = 0; k < 4; ++k) sm.x[hh * 64 + d0 + k] = round_bf16(o[k] * inv);
      }
      consumer_sync<kConsumers>();
      load_x<S, S::KD>(sm.x, xr);
    }
    // ---- O rows: HM = H + attn @ Wo^T ----
    {
      const int a = split_begin(cta, S::D, G), b = split_begin(cta + 1, S::D, G);
      ok = gemv_phase<S::KD, S::ROWB_D, false>(A, ring, flag, t0, a, b, S::RPS_D, xr,
                                               [&](int u, float v, float) {
                                                 if (lane == 0) st_word(lw + A.w_hm + u, sm.h[u] + v, flag);
                                               });
      ok = consumer_sync_and<kConsumers>(ok);
      if (!ok) break;
    }
    // ---- gather HM (the residual after attention) ----
    ok = gather_pairs<(S::D / 2 + kConsumers - 1) / kConsumers>(
        A, flag, t0, SITE_HM, [&](int i) { return lw + A.w_hm + 2 * (t + i * kConsumers); },
        [&](int i) { return t + i * kConsumers < S::D / 2; },
        [&](int i, float a, float b) { const int k = t + i * kConsumers; sm.h[2 * k] = a; sm.h[2 * k + 1] = b; });
    ok = consumer_sync_and<kConsumers>(ok);
    if (!ok) break;
    rmsnorm_to_x<S>(sm, A.ln2 + static_cast<size_t>(l) * S::D, A.eps);
    load_x<S, S::KD>(sm.x, xr);
    // ---- gate/up pairs -> act = silu(g) * u ----
    {
      const int a = split_begin(cta, S::DFF, G), b = split_begin(cta + 1, S::DFF, G);
      ok = gemv_phase<S::KD, S::ROWB_D, true>(A, ring, flag, t0, a, b, S::PPS, xr,
                                              [&](int u, float gt, float up) {
                                                if (lane == 0) {
                                                  const float act = gt * (1.0f / (1.0f + __expf(-gt))) * up;
                                                  st_word(lw + A.w_act + u, act, flag);
                                                }
                                              });
      ok = consumer_sync_and<kConsumers>(ok);
      if (!ok) break;
    }
    // ---- gather act -> x (bf16), down rows: H_{l+1} = HM + act @ Wd^T ----
    {
      ok = gather_pairs<(S::DFF / 2 + kConsumers - 1) / kConsumers>(
          A, flag, t0, SITE_ACT, [&](int i) { return lw + A.w_act + 2 * (t + i * kConsumers); },
          [&](int i) { return t + i * kConsumers < S::DFF / 2; },
          [&](int i, float a, float b) {
            const int k = t + i * kConsumers;
            sm.x[2 * k] = round_bf16(a);
            sm.x[2 * k + 1] = round_bf16(b);
          });
      ok = consumer_sync_and<kConsumers>(ok);
      if (!ok) break;
      uint4 xf[S::KF];
      load_x<S, S::KF>(sm.x, xf);
      uint64_t* nxt = A.words + static_cast<size_t>(l + 1) * A.layer_words;  // H_{l+1} at word 0
      const int a = split_begin(cta, S::D, G), b = split_begin(cta + 1, S::D, G);
      ok = gemv_phase<S::KF, S::ROWB_F, false>(A, ring, flag, t0, a, b, S::RPS_F, xf,
                                               [&](int u, float v, float) {
                                                 if (lane == 0) st_word(nxt + u, sm.h[u] + v, flag);
                                               });
      ok = consumer_sync_and<kConsumers>(ok);
      if (!ok) break;
    }
  }

  if (ok) {
    // ---- final norm + tied logits + argmax (reference :314-357) ----
    uint64_t* fw = A.words + static_cast<size_t>(A.n_layers) * A.layer_words;
    ok = gather_pairs<(S::D / 2 + kConsumers - 1) / kConsumers>(
        A, flag, t0, SITE_FINAL, [&](int i) { return fw + 2 * (t + i * kConsumers); },
        [&](int i) { return t + i * kConsumers < S::D / 2; },
        [&](int i, float a, float b) { const int k = t + i * kConsumers; sm.h[2 * k] = a; sm.h[2 * k + 1] = b; });
    ok = consumer_sync_and<kConsumers>(ok);
  }
  if (ok) {
    rmsnorm_to_x<S>(sm, A.lnf, A.eps);
    load_x<S, S::KD>(sm.x, xr);
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const int a = split_begin(cta, A.vocab, G), b = split_begin(cta + 1, A.vocab, G);
    ok = gemv_phase<S::KD, S::ROWB_D, false>(A, ring, flag, t0, a, b, S::RPS_D, xr,
                                             [&](int u, float v, float) {
                                               if (lane == 0 && A.logits) A.logits[u] = v;
                                               if (v > best_v) { best_v = v; best_i = u; }
                                             });
    ok = consumer_sync_and<kConsumers>(ok);
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
          *A.next_tok = gi == 0x7fffffff ? 0 : gi;
          A.ctl->arrive = 0u;
          __threadfence();
          st_relaxed_u32(&A.ctl->gen, flag);
        }
      }
    }
  }
  if (!ok) {
    *reinterpret_cast<volatile int*>(&sm.abort) = 1;
  }
}

}  // namespace b2d
