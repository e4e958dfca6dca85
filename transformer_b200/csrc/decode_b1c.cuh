// decode_b1c.cuh — the B=1 decode step on thread-block clusters (sm_100a).
//
// Same step, same math references as decode_b1.cuh (kernels/multi_sm_decode.py
// :35-357), with the layer's communication restructured around clusters of
// kCS CTAs so that a layer needs two grid-wide exchanges instead of five:
//
//  * cluster c < n_heads owns attention head c.  Its CTAs compute the head's
//    q rows and its kv group's k / v rows (16 rows each per CTA), push them to
//    every CTA of the cluster through distributed shared memory, each run the
//    attention over a quarter of the positions, push their (o, m, l) partials
//    the same way and merge them in a fixed order.  No grid-wide exchange.
//  * O projection, split over K: CTA k of head cluster h multiplies rows
//    [k D/kCS, (k+1) D/kCS) of Wo's 64 columns of head h (a 2D tensor copy of
//    the weight as stored) by the head's output and adds the products to the
//    residual accumulators HM (one contribution per head per element).
//  * gate/up rows of act chunks (8 SwiGLU units) split over all CTAs; the CTA
//    keeps its acts and multiplies them by Wd's matching 8-column blocks
//    (tensor copies of the weight as stored): a partial of every output.  The
//    cluster sums its partials over distributed shared memory (CTA k sums
//    rows [k D/kCS, ...)) and adds the sums to the accumulators H_{l+1} (one
//    contribution per cluster per element).
//  * residual accumulators are exact fixed-point words (b2d_ptx.cuh): the
//    adds land in any order and give the same bits; a reader waits until a
//    word's count reaches the number of contributors.  Each step uses one of
//    two accumulator sets (by flag parity) and zeroes the other for the next
//    step, so no memset runs between launches.
//  * cluster signalling: a CTA pushes with st.async, which completes bytes of
//    a transaction on the receiver's mbarrier; the receiver arms the phase
//    with the bytes it expects and waits with a bounded poll.  One mbarrier
//    per purpose, each used once per layer; every CTA of the cluster pushes to
//    every CTA in each of them, so a sender always waits for its receivers'
//    pushes of the same phase before it can finish.  A failed wait makes the
//    CTA skip the rest of its work but keep its schedule, and every CTA ends
//    with a cluster barrier, so no CTA exits while a peer may still address
//    its shared memory.
//  * weights stream through a producer-warp ring as in decode_b1.cuh, but
//    every stage is ONE tensor copy of 16 KB: gate/up and q/k/v rows arrive as
//    [K/64 k-blocks][rows][64] with the 128-byte swizzle (conflict-free
//    ldmatrix without padded rows), Wo and Wd blocks as described above.  The
//    producer never waits on activations.
#pragma once

#include "decode_b1.cuh"
#include "tc_ptx.cuh"

namespace b2d {

constexpr int kCS = 4;            // CTAs per cluster
constexpr int kMinGridC = 120;    // fewest CTAs the per-CTA budgets assume
// Act chunks are split over the CTAs in proportion to a weight:
// kChunkWeightHead for a CTA of a head cluster (which also streams 48 q/k/v
// rows and a Wo block per layer), kChunkWeightOther for the others.  Measured
// at 132 CTAs: 1 : 3 (head CTAs 1-2 chunks, others 3-4) 266 us/token; 4 : 5
// (at most 3 chunks everywhere) 316 us: a head CTA with 3 chunks no longer
// fits its layer in the weight ring and waits for its down stages.
constexpr int kChunkWeightHead = 1, kChunkWeightOther = 3;
constexpr int kMaxChunksC = 4;    // act chunks per CTA at most (the host checks its grid against it)
// Weight ring: every stage is one 16 KB tensor copy, so 12 of them fit.
constexpr int kStagesC = 12;
constexpr int kStageBytesC = 16384;
using RingC = RingT<kStagesC, kStageBytesC>;
constexpr int kAttRows = 64;      // K/V positions staged per attention pass
enum : uint32_t {
  ST_RANGE = 0x300u,              // | site: a residual contribution out of the accumulator range
  SITE_QKVX = 12, SITE_ATTX = 13, SITE_DRED = 14,
};

template <class S>
struct ShapeC {
  static constexpr int QROWS = 64 / kCS;                    // q (and k, v) rows per CTA of a head cluster
  static constexpr int QKV_ROWS = 3 * QROWS;
  static constexpr int OROWS = S::D / kCS;                  // residual rows a cluster CTA owns
  static constexpr int OBOX = OROWS < 128 ? OROWS : 128;    // Wo rows per tensor copy (one stage)
  static constexpr int OBOXES = OROWS / OBOX;
  static constexpr int CHUNKS = S::DFF / 8;                 // act chunks of 8 units
  static constexpr int MAXCH = kMaxChunksC;
  static constexpr int GU_ROWS = 16 * MAXCH;
  static constexpr int DBOX = S::D < 256 ? S::D : 256;      // Wd rows per tensor copy
  static constexpr int DBOXES = S::D / DBOX;
  static constexpr int PS = kStageBytesC / S::ROWB_D;       // K = D rows per stage (k-block layout; logits)
  static constexpr int QPS = QROWS < PS ? QROWS : PS;       // rows per stage of the q / k / v ranges
  static constexpr int MT_QKV = (QKV_ROWS + 15) / 16, MT_GU = (GU_ROWS + 15) / 16;
  static constexpr int MT_MAX = MT_QKV > MT_GU ? MT_QKV : MT_GU;
  static_assert(64 % kCS == 0 && QROWS % QPS == 0, "q/k/v rows fill whole stages");
  static_assert(OROWS % 16 == 0 && OROWS % OBOX == 0 && OBOX * 128 <= kStageBytesC, "Wo boxes");
  static_assert(S::D % DBOX == 0 && S::D * 16 <= kStageBytesC, "one act chunk's Wd columns fill one stage");
  static_assert(S::D % 64 == 0 && PS >= 1 && PS * S::ROWB_D <= kStageBytesC, "k-block stages");
  static_assert(S::DFF % 8 == 0 && 2 * MAXCH <= kStagesC, "gate/up stages resident together");
  static_assert(S::D / 4 <= kConsumers && OROWS <= kConsumers, "one thread per pushed quad / owned row");
  static_assert(S::GQA * S::NKV == S::NH, "GQA");
  // bytes each CTA receives per layer through each cluster barrier
  static constexpr uint32_t kQkvBytes = kCS * QKV_ROWS * 4;
  static constexpr uint32_t kAttpBytes = kCS * (32 * 8 + 8);
  static constexpr uint32_t kDredBytes = S::D * 4;
};

template <class S>
struct SmemC {
  using C = ShapeC<S>;
  alignas(1024) uint8_t stage[kStagesC][kStageBytesC];
  uint64_t full[kStagesC];
  uint64_t empty[kStagesC];
  uint64_t qkv_bar;   // q/k/v pushes of the cluster (kQkvBytes per layer)
  uint64_t attp_bar;  // attention partial pushes (kAttpBytes)
  uint64_t dred_bar;  // down partial pushes (kDredBytes)
  alignas(16) __nv_bfloat16 xb[S::D];          // GEMV input (bf16)
  // The attention's K/V rows and the MLP's down partials are never live at
  // once: a peer pushes its down partials only after this CTA's attention of
  // the layer fed the HM accumulators it waited for, and the next layer's K/V
  // copies start after the barrier that ends this layer.
  union alignas(128) {
    struct {  // K/V rows of one pass: row r's 16-byte chunk c at r * 128 + ((c ^ (r & 7)) << 4)
      __nv_bfloat16 k[kAttRows][64];
      __nv_bfloat16 v[kAttRows][64];
    } att;
    struct {
      float pd[S::D];               // this CTA's down partial
      float pr[kCS][C::OROWS];      // the cluster's down partials of this CTA's rows
    } dn;
  } u;
  alignas(16) float qkv[3 * 64];               // head q, kv-group k, v (pushed by the cluster)
  alignas(16) float rq[64];
  alignas(16) float rk[64];
  float wo[kConsumerWarps][64];
  float wm[kConsumerWarps], wl[kConsumerWarps];
  float red[kConsumerWarps];
  alignas(16) float attp[kCS][68];             // attention partials (o[64], m, l) by sender rank
  int64_t fix[C::OROWS];                       // exact residual sums of this CTA's rows (cluster 0)
  float act[8 * C::MAXCH];
  float part[kConsumerWarps][C::MT_MAX * 16];
  float am_v[kConsumerWarps];
  int am_i[kConsumerWarps];
  int abort;
  int tok_in;
};
template <class S>
constexpr size_t smem_c_bytes() { return sizeof(SmemC<S>) + 1024; }  // + base alignment
template <class S>
struct SmemCChecks {
  static_assert(offsetof(SmemC<S>, stage) == 0, "stages first (1024-aligned base)");
  static_assert(offsetof(SmemC<S>, xb) % 16 == 0 && offsetof(SmemC<S>, u) % 128 == 0 &&
                offsetof(SmemC<S>, attp) % 16 == 0, "vector fields");
  static_assert(offsetof(SmemC<S>, full) % 8 == 0, "mbarriers");
  static_assert(smem_c_bytes<S>() <= 232448, "shared memory per CTA");
  static constexpr bool ok = true;
};

// First act chunk of CTA c when G CTAs share the CHUNKS chunks (weights as
// above; CTAs c >= gridDim.x exist only in the failure-injection test).
template <class S>
__device__ __host__ __forceinline__ int chunk_begin(int c, int G) {
  const int nh = S::NH * kCS;
  const auto w = [nh](int x) {
    return static_cast<long long>(x <= nh ? kChunkWeightHead * x
                                          : kChunkWeightHead * nh + kChunkWeightOther * (x - nh));
  };
  return static_cast<int>(static_cast<long long>(ShapeC<S>::CHUNKS) * w(c) / w(G));
}

// Accumulator words of a residual vector after sublayer `which` (0 = HM_l,
// after attention; 1 = H_{l+1}, after the MLP) of layer l, parity `par`.
// Element r's word sits at r * kAccStride.  Packed (1) is faster than one
// word per 32-byte sector (4): measured, the polls of 4x the sectors cost
// more than the atomic adds gain.
constexpr int kAccStride = 1;
__device__ __forceinline__ uint64_t* acc_word(const DecodeArgs& A, uint32_t par, int l, int which, int d) {
  return A.acc + (static_cast<size_t>(par) * A.n_layers * 2 + static_cast<size_t>(2 * l + which)) * d * kAccStride;
}
// The words of elements 2i and 2i + 1.
__device__ __forceinline__ void acc_ld2(const uint64_t* v, int i, uint64_t& a, uint64_t& b) {
  if constexpr (kAccStride == 1) {
    ld_words2(v + 2 * i, a, b);  // one 16-byte load
  } else {
    a = ld_relaxed_u64(v + 2 * i * kAccStride);
    b = ld_relaxed_u64(v + (2 * i + 1) * kAccStride);
  }
}

// Waits until every word of a residual vector (D accumulator words at src)
// holds `target` contributions; thread t takes the word pairs (2m, 2m + 1),
// m = t + kConsumers i, into hv as f32 and hands the exact sums to
// keep(row, sum_row, sum_row+1).  Returns false on timeout / abort.
template <class S, int NP, class KeepF>
__device__ __forceinline__ bool gather_acc(const DecodeArgs& A, const uint64_t* src, uint32_t target, uint32_t flag,
                                           uint64_t t0, uint32_t site, float (&hv)[NP][2], KeepF keep) {
  const int t = threadIdx.x;
  uint32_t pending = 0;
#pragma unroll
  for (int i = 0; i < NP; ++i)
    if (t + i * kConsumers < S::D / 2) pending |= 1u << i;
  Waiter wt;
  while (true) {
    uint64_t a[NP], b[NP];
#pragma unroll
    for (int i = 0; i < NP; ++i)
      if (pending & (1u << i)) acc_ld2(src, t + i * kConsumers, a[i], b[i]);
#pragma unroll
    for (int i = 0; i < NP; ++i) {
      if ((pending & (1u << i)) && acc_count(a[i]) == target && acc_count(b[i]) == target) {
        const int64_t sa = acc_sum(a[i], target), sb = acc_sum(b[i], target);
        hv[i][0] = acc_value(sa);
        hv[i][1] = acc_value(sb);
        keep(2 * (t + i * kConsumers), sa, sb);
        pending &= ~(1u << i);
      }
    }
    if (!pending) return true;
    if (A.poll_ns) __nanosleep(A.poll_ns);
    if (wt.expired(A, flag, t0, site)) return false;
  }
}

// x = bf16(h * rsqrt(mean(h^2) + eps) * g) into sm.xb (RMSNorm, reference
// :121-126) from the residual pairs in hv.  `ok` enters the first barrier's AND.
template <class S, int NP>
__device__ __forceinline__ bool norm_x(SmemC<S>& sm, const float (&hv)[NP][2], const float2 (&g)[NP], float eps,
                                       bool ok) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < NP; ++i) {
    if (t + i * kConsumers < S::D / 2) {
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

// Bounded wait (every consumer thread) for phase `parity` of a cluster
// signalling mbarrier.
__device__ __forceinline__ bool wait_cluster_bar(const DecodeArgs& A, uint64_t* bar, uint32_t parity, uint32_t flag,
                                                 uint64_t t0, uint32_t site) {
  Waiter wt;
  while (!mbar_test_cluster(bar, parity)) {
    if (wt.expired(A, flag, t0, site)) return false;
  }
  return true;
}

// Raises ST_RANGE (first error wins) for a contribution out of range.
__device__ __forceinline__ bool acc_contrib(const DecodeArgs& A, float v, int64_t base, uint32_t flag, uint32_t site,
                                            int64_t& q) {
  int64_t f;
  const bool in = acc_fix(v, f);
  q = f + base;
  if (!in || q >= static_cast<int64_t>(kAccBias) || q <= -static_cast<int64_t>(kAccBias)) {
    raise_error(A.ctl, ST_RANGE | site, flag);
    q = 0;
    return false;
  }
  return true;
}

// Producer warp: streams this CTA's weights for every step, in the order the
// consumers take them: per layer [q, k, v rows; Wo boxes] (head clusters),
// gate/up rows, Wd column blocks; then the logits rows.
// The cluster kernel's weight views (kernel parameters).
struct MapsC {
  CUtensorMap qkv;   // {64, QKV rows, D/64, L}, box {64, QPS, D/64, 1}, 128-byte swizzle
  CUtensorMap o;     // {D, D, L}, box {64, OBOX, 1}, 128-byte swizzle
  CUtensorMap gu;    // {64, 2 DFF rows, D/64, L}, box {64, PS, D/64, 1}, 128-byte swizzle
  CUtensorMap down;  // {DFF, D, L}, box {8, DBOX, 1}
};

template <class S, bool TR>
__device__ void producer_c(const DecodeArgs& A, SmemC<S>& sm, const MapsC& maps, int cta, int head, int rank, int a8,
                           int nch, int v0, int v1, uint32_t flag, uint64_t t0, int nsteps) {
  using C = ShapeC<S>;
  const int lane = threadIdx.x & 31;
  const uint64_t pol = l2_policy_evict_first();
  uint32_t seq = 0, landed = 0;
  const uint32_t cap = static_cast<uint32_t>(A.max_inflight);
  bool ok = true;
  // Arms the next ring slot for `bytes` (warp-uniform); -1 when the launch aborted.
  auto arm = [&](uint32_t bytes) -> int {
    const uint32_t slot = seq % kStagesC;
    bool good = true;
    if (lane == 0) {
      while (good && seq - landed >= cap) {
        ProducerWaiter wt;
        while (!mbar_test(&sm.full[landed % kStagesC], (landed / kStagesC) & 1u)) {
          if (*reinterpret_cast<volatile int*>(&sm.abort) || wt.expired(A, flag, t0, SITE_FULL)) {
            good = false;
            break;
          }
        }
        if (good) ++landed;
      }
      if (good && seq >= kStagesC) {
        const uint32_t par = ((seq / kStagesC) - 1) & 1u;
        ProducerWaiter wt;
        while (!mbar_test(&sm.empty[slot], par)) {
          if (*reinterpret_cast<volatile int*>(&sm.abort) || wt.expired(A, flag, t0, SITE_EMPTY)) {
            good = false;
            break;
          }
        }
      }
      if (good) mbar_arrive_expect_tx(&sm.full[slot], bytes);
    }
    if (!__shfl_sync(0xffffffffu, good ? 1 : 0, 0)) {
      ok = false;
      return -1;
    }
    if (lane == 0) stage_stamp<TR>(A, cta, 0, seq);
    ++seq;
    return static_cast<int>(slot);
  };
  // n rows of K = D from src (the logits), `per` rows per stage, one copy each.
  auto rows = [&](const uint8_t* src, int n, int per) {
    for (int u = 0; u < n && ok; u += per) {
      const int cnt = min(per, n - u);
      const int slot = arm(static_cast<uint32_t>(cnt) * S::ROWB_D);
      if (slot >= 0 && lane == 0)
        bulk_g2s(sm.stage[slot], src + static_cast<size_t>(u) * S::ROWB_D, static_cast<uint32_t>(cnt) * S::ROWB_D,
                 &sm.full[slot], pol);
    }
  };
  for (int step = 0; step < nsteps && ok; ++step) {
    for (int l = 0; l < A.n_layers && ok; ++l) {
      if (head >= 0) {
        const int g = head / S::GQA;
        const int r0[3] = {64 * head, S::NH * 64 + 64 * g, (S::NH + S::NKV) * 64 + 64 * g};
        for (int comp = 0; comp < 3; ++comp) {
          for (int u = 0; u < C::QROWS && ok; u += C::QPS) {
            const int slot = arm(C::QPS * S::ROWB_D);
            if (slot >= 0 && lane == 0)
              tma_load_4d(sm.stage[slot], &maps.qkv, 0, r0[comp] + rank * C::QROWS + u, 0, l, &sm.full[slot], pol);
          }
        }
        for (int b = 0; b < C::OBOXES && ok; ++b) {
          const int slot = arm(C::OBOX * 128);
          if (slot >= 0 && lane == 0)
            tma_load_3d(sm.stage[slot], &maps.o, 64 * head, rank * C::OROWS + b * C::OBOX, l, &sm.full[slot], pol);
        }
      }
      for (int u = 0; u < 16 * nch && ok; u += C::PS) {  // a box past the CTA's rows brings rows it ignores
        const int slot = arm(C::PS * S::ROWB_D);
        if (slot >= 0 && lane == 0) tma_load_4d(sm.stage[slot], &maps.gu, 0, 16 * a8 + u, 0, l, &sm.full[slot], pol);
      }
      for (int ch = 0; ch < nch && ok; ++ch) {
        const int slot = arm(S::D * 16);
        if (slot >= 0 && lane == 0) {
          for (int b = 0; b < C::DBOXES; ++b)
            tma_load_3d(sm.stage[slot] + b * C::DBOX * 16, &maps.down, 8 * (a8 + ch), b * C::DBOX, l, &sm.full[slot],
                        pol);
        }
      }
    }
    if (ok) rows(A.wbase + A.off_emb + static_cast<size_t>(v0) * S::ROWB_D, v1 - v0, C::PS);
  }
  if (lane == 0) {
    // never leave with copies in flight (bounded)
    const uint32_t first = seq > kStagesC ? seq - kStagesC : 0;
    const uint64_t td = globaltimer_ns();
    for (uint32_t s = first; s < seq; ++s) {
      while (!mbar_test(&sm.full[s % kStagesC], (s / kStagesC) & 1u)) {
        if (globaltimer_ns() - td > A.wait_ns) break;
      }
    }
  }
}

// K/V staging of one attention pass: cached positions [base, min(base +
// kAttRows, p1, pos)) of kv head g, layer l, into sm.u.att by 16-byte cp.async
// copies from every consumer thread (row r's chunk c at r * 128 + ((c ^ (r &
// 7)) << 4)).  They bypass the tensor-copy unit, whose queue holds the weight
// stream.  Each thread waits for its own copies (cp.async.wait_all) before the
// barrier that publishes them.
template <class S>
__device__ __forceinline__ void att_issue_c(const DecodeArgs& A, SmemC<S>& sm, int l, int g, int pos, int base,
                                            int p1) {
  const size_t half = static_cast<size_t>(S::NKV) * A.ctx * S::DH;
  const __nv_bfloat16* Kc = A.kv + static_cast<size_t>(l) * 2 * half + static_cast<size_t>(g) * A.ctx * S::DH +
                            static_cast<size_t>(base) * S::DH;
  const int ncached = max(0, min(min(base + kAttRows, p1), pos) - base);
  for (int i = threadIdx.x; i < ncached * 8; i += kConsumers) {  // 8 chunks of 16 bytes per row
    const int r = i >> 3, c = i & 7;
    const int off = r * 64 + ((c ^ (r & 7)) << 3);
    cp_async16(&sm.u.att.k[0][0] + off, Kc + 8 * i);
    cp_async16(&sm.u.att.v[0][0] + off, Kc + half + 8 * i);
  }
  cp_async_commit();
}

// K (kv = 0) or V (kv = 1) rows of a later attention pass, issued by the
// warp that reads them: each warp owns rows [8 warp, 8 warp + 8) of a pass
// (positions base + row), so its next pass's rows can be loaded as soon as it
// has read the current ones, with no block barrier.  One cp.async group.
template <class S>
__device__ __forceinline__ void att_issue_warp(const DecodeArgs& A, SmemC<S>& sm, int l, int g, int pos, int base,
                                               int p1, int kv) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const size_t half = static_cast<size_t>(S::NKV) * A.ctx * S::DH;
  const __nv_bfloat16* src = A.kv + static_cast<size_t>(l) * 2 * half + (kv ? half : 0) +
                             static_cast<size_t>(g) * A.ctx * S::DH;
  __nv_bfloat16* dst = kv ? &sm.u.att.v[0][0] : &sm.u.att.k[0][0];
  const int lim = min(p1, pos);  // position pos comes from the new K / V, not the cache
#pragma unroll
  for (int k = 0; k < 2; ++k) {  // 8 rows x 8 chunks of 16 bytes per warp
    const int i = lane + 32 * k, r = warp * 8 + (i >> 3), c = i & 7;
    if (base + r < lim) cp_async16(dst + r * 64 + ((c ^ (r & 7)) << 3), src + static_cast<size_t>(base + r) * S::DH + 8 * c);
  }
  cp_async_commit();
}

// One attention pass over positions [base, base + kAttRows) of [p0, p1),
// accumulated into (m, lsum, o0, o1) (online softmax).  MULTI (the slice
// needs more than one pass): every warp loads its own rows of the next pass
// as soon as it has read the current ones (att_issue_warp), with no block
// barrier between passes.  The single-pass form keeps its original schedule
// (the multi-pass form measured ~2 us/token slower on single-pass slices).
template <class S, bool TR, bool MULTI>
__device__ __forceinline__ void att_pass(const DecodeArgs& A, SmemC<S>& sm, int l, int g, int pos, int base, int p0,
                                         int p1, const float (&qv)[16], float vn0, float vn1, float& m, float& lsum,
                                         float& o0, float& o1, int ts) {
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int qi = lane >> 2, q4 = lane & 3;  // position within the warp's 8, dim quarter
  const bool more = MULTI && base + kAttRows < p1;  // a later pass follows
  if (MULTI && base != p0) {  // this warp's K rows of the pass (its V rows may still be in flight)
    cp_async_wait<1>();
    __syncwarp();
  }
  const int r = warp * 8 + qi, pk = base + r;
  float sa = 0.f, sb = 0.f;
  if (pk == pos) {
#pragma unroll
    for (int d = 0; d < 16; d += 2) {
      sa = fmaf(qv[d], sm.rk[16 * q4 + d], sa);
      sb = fmaf(qv[d + 1], sm.rk[16 * q4 + d + 1], sb);
    }
  } else if (pk < p1) {
    const uint4* kr = reinterpret_cast<const uint4*>(sm.u.att.k[r]);
    const uint4 k0 = kr[(2 * q4) ^ qi], k1 = kr[(2 * q4 + 1) ^ qi];  // (r & 7) == qi
    sa = fmaf(qv[0], bf16_lo(k0.x), sa);
    sb = fmaf(qv[1], bf16_hi(k0.x), sb);
    sa = fmaf(qv[2], bf16_lo(k0.y), sa);
    sb = fmaf(qv[3], bf16_hi(k0.y), sb);
    sa = fmaf(qv[4], bf16_lo(k0.z), sa);
    sb = fmaf(qv[5], bf16_hi(k0.z), sb);
    sa = fmaf(qv[6], bf16_lo(k0.w), sa);
    sb = fmaf(qv[7], bf16_hi(k0.w), sb);
    sa = fmaf(qv[8], bf16_lo(k1.x), sa);
    sb = fmaf(qv[9], bf16_hi(k1.x), sb);
    sa = fmaf(qv[10], bf16_lo(k1.y), sa);
    sb = fmaf(qv[11], bf16_hi(k1.y), sb);
    sa = fmaf(qv[12], bf16_lo(k1.z), sa);
    sb = fmaf(qv[13], bf16_hi(k1.z), sb);
    sa = fmaf(qv[14], bf16_lo(k1.w), sa);
    sb = fmaf(qv[15], bf16_hi(k1.w), sb);
  }
  float sdot = sa + sb;
  sdot += __shfl_xor_sync(0xffffffffu, sdot, 1);
  sdot += __shfl_xor_sync(0xffffffffu, sdot, 2);
  if (more) {  // every lane has read its K row: the next pass's K rows replace them
    __syncwarp();
    att_issue_warp<S>(A, sm, l, g, pos, base + kAttRows, p1, 0);
  }
  const bool valid = pk < p1;
  const float s = valid ? sdot : -INFINITY;
  float mx = s;
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float mn = fmaxf(m, mx);
  const float pe = valid ? __expf(s - mn) : 0.f;
  float ps = pe;
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
  const float alpha = m == -INFINITY ? 0.f : __expf(m - mn);
  if (q4 == 0) sm.wo[warp][qi] = pe;  // stage probabilities for PV
  __syncwarp();
  if (base == p0) trace_stamp<TR>(A, ts + 11);
  if (MULTI && base != p0) {  // this warp's V rows of the pass (the next pass's K rows may be in flight)
    if (more) cp_async_wait<1>(); else cp_async_wait<0>();
    __syncwarp();
  }
  float a0 = 0.f, a1 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int rv = warp * 8 + i, pv = base + rv;
    const float pi = sm.wo[warp][i];
    float v0 = 0.f, v1 = 0.f;
    if (pv == pos) {
      v0 = vn0;
      v1 = vn1;
    } else if (pv < p1) {
      const uint32_t vw =
          reinterpret_cast<const uint32_t*>(sm.u.att.v[rv])[(((lane >> 2) ^ (rv & 7)) << 2) + (lane & 3)];
      v0 = bf16_lo(vw);
      v1 = bf16_hi(vw);
    }
    a0 = fmaf(pi, v0, a0);
    a1 = fmaf(pi, v1, a1);
  }
  __syncwarp();
  if (more) att_issue_warp<S>(A, sm, l, g, pos, base + kAttRows, p1, 1);  // every lane has read its V rows
  lsum = fmaf(lsum, alpha, ps);
  o0 = fmaf(o0, alpha, a0);
  o1 = fmaf(o1, alpha, a1);
  m = mn;
  if (!MULTI) consumer_sync<kConsumers>();  // staged K/V read by every warp before the union is reused
}

// The attention of head h over this CTA's positions [p0, p1) (reference
// :182-221), from q/k/v in sm.qkv: RoPE, then passes of kAttRows positions.
// A warp owns 8 positions of a pass, four lanes per position (16 dims each),
// so a score is a 16-term dot product and two shuffles; online softmax per
// warp; PV with lane l on dims 2l, 2l + 1.  Returns the unnormalised partial
// in warp 0's registers: lane l holds o[2l], o[2l + 1] in (b0, b1), and M, L.
// The K/V rows of the first pass were issued with the layer (att_issue_c).
template <class S, bool TR>
__device__ __forceinline__ void attention_slice(const DecodeArgs& A, SmemC<S>& sm, int l, int pos, int h, int p0,
                                                int p1, float rc, float rs, float& b0, float& b1, float& Mo,
                                                float& Lo, int ts) {
  static_assert(kAttRows == 8 * kConsumerWarps, "a pass is 8 positions per warp");
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int g = h / S::GQA;
  const int qi = lane >> 2, q4 = lane & 3;  // position within the warp's 8, dim quarter
  cp_async_wait_all();  // this thread's share of the first pass's K/V rows (issued with the layer)
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
  trace_stamp<TR>(A, ts + 10);
  float qv[16];
#pragma unroll
  for (int d = 0; d < 16; ++d) qv[d] = sm.rq[16 * q4 + d];
  const float vn0 = sm.qkv[128 + 2 * lane], vn1 = sm.qkv[128 + 2 * lane + 1];
  float m = -INFINITY, lsum = 0.f, o0 = 0.f, o1 = 0.f;
  if (p1 - p0 <= kAttRows) {
    if (p0 < p1) att_pass<S, TR, false>(A, sm, l, g, pos, p0, p0, p1, qv, vn0, vn1, m, lsum, o0, o1, ts);
  } else {
    for (int base = p0; base < p1; base += kAttRows)
      att_pass<S, TR, true>(A, sm, l, g, pos, base, p0, p1, qv, vn0, vn1, m, lsum, o0, o1, ts);
  }
  trace_stamp<TR>(A, ts + 12);
  sm.wo[warp][2 * lane] = o0;
  sm.wo[warp][2 * lane + 1] = o1;
  if (lane == 0) {
    sm.wm[warp] = m;
    sm.wl[warp] = lsum;
  }
  consumer_sync<kConsumers>();
  if (warp == 0) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) M = fmaxf(M, sm.wm[w]);
    float L = 0.f, c0 = 0.f, c1 = 0.f;
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) {
      const float e = sm.wl[w] > 0.f ? __expf(sm.wm[w] - M) : 0.f;
      L = fmaf(sm.wl[w], e, L);
      c0 = fmaf(sm.wo[w][2 * lane], e, c0);
      c1 = fmaf(sm.wo[w][2 * lane + 1], e, c1);
    }
    b0 = c0;
    b1 = c1;
    Mo = M;
    Lo = L;
  }
  // The first head of the group appends this position's K (post-RoPE) and V
  // to the cache in bf16 (the CTA whose positions include pos).
  if (warp == 1 && (h % S::GQA) == 0 && pos >= p0 && pos < p1) {
    const size_t half = static_cast<size_t>(S::NKV) * A.ctx * S::DH;
    __nv_bfloat16* kd = A.kv + static_cast<size_t>(l) * 2 * half + static_cast<size_t>(g) * A.ctx * S::DH +
                        static_cast<size_t>(pos) * S::DH;
    reinterpret_cast<__nv_bfloat162*>(kd)[lane] = __floats2bfloat162_rn(sm.rk[2 * lane], sm.rk[2 * lane + 1]);
    reinterpret_cast<__nv_bfloat162*>(kd + half)[lane] = __floats2bfloat162_rn(vn0, vn1);
  }
  consumer_sync<kConsumers>();  // wo / wm / wl free again
}

// One GEMV phase over `rows` weight rows on warp-level tensor-core MMAs, like
// gemv_phase (decode_b1.cuh) but reading k-block stages: a stage holds RB
// consecutive rows as [K/64][RB][64] bf16 with the 128-byte swizzle (16-byte
// chunk c of row r at ((c ^ (r & 7)) << 4) within the row's 128 bytes).
// Warp w takes K slice [w K/8, (w+1) K/8) of every 16-row tile that holds
// rows; the input fragments of the whole slice are loaded first and the
// weight fragments one K step ahead of their MMAs (ldmatrix latency is ~100
// cycles).  Thread r sums the warps' partials in warp order and calls
// out(r, v); with SWIGLU, rows (2j, 2j + 1) are gate and up of unit j and
// out(j, silu(gate) * up) is called instead.  Returns the AND of every
// warp's waits (after the phase's closing barrier).
template <int K, int RB, int MT, int PSTRIDE, bool TR, bool SWIGLU, class Out>
__device__ __forceinline__ bool gemv_phase_sw(const DecodeArgs& A, RingC& ring, float* part, const __nv_bfloat16* xb,
                                              uint32_t flag, uint64_t t0, int rows, Out out) {
  static_assert(MT * 16 <= PSTRIDE, "partial buffer");
  constexpr int KS = K / 16 / kConsumerWarps;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int ns = rows > 0 ? (rows + RB - 1) / RB : 0;
  bool ok = rows <= MT * 16 && ns <= kStagesC;
  if (ok && ns > 0) ok = wait_full_n(A, ring, ns, flag, t0);
  if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 1, ring.seq);
  if (ok && rows > 0) {
    const int nt = (rows + 15) >> 4;  // tiles holding rows
    const int lr = (lane & 7) + 8 * ((lane >> 3) & 1), lk = 8 * (lane >> 4);
    uint32_t rbase[MT];
    uint32_t rsw[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int r = min(mt * 16 + lr, rows - 1);  // rows past the range: any valid row
      const int st = r / RB, rr = r - st * RB;
      rbase[mt] = smem_addr(ring.stage[(ring.seq + static_cast<uint32_t>(st)) % kStagesC]) +
                  static_cast<uint32_t>(rr * 128);
      rsw[mt] = static_cast<uint32_t>(rr & 7);
    }
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(xb);
    const int k0 = warp * KS * 16;
    uint32_t bx[KS][2];
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      bx[s][0] = x32[(k0 + 16 * s + 2 * tig) >> 1];
      bx[s][1] = x32[(k0 + 16 * s + 8 + 2 * tig) >> 1];
    }
    auto a_addr = [&](int mt, int s) {
      const int kl = k0 + 16 * s + lk;
      return rbase[mt] + static_cast<uint32_t>((kl >> 6) * RB * 128) +
             ((static_cast<uint32_t>((kl >> 3) & 7) ^ rsw[mt]) << 4);
    };
    float acc[MT][4];
    uint32_t af[2][MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
      if (mt < nt) ldsm_x4(a_addr(mt, 0), af[0][mt][0], af[0][mt][1], af[0][mt][2], af[0][mt][3]);
    }
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      if (s + 1 < KS) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          if (mt < nt)
            ldsm_x4(a_addr(mt, s + 1), af[(s + 1) & 1][mt][0], af[(s + 1) & 1][mt][1], af[(s + 1) & 1][mt][2],
                    af[(s + 1) & 1][mt][3]);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        if (mt < nt)
          mma_bf16(acc[mt], af[s & 1][mt][0], af[s & 1][mt][1], af[s & 1][mt][2], af[s & 1][mt][3], bx[s][0],
                   bx[s][1]);
    }
    if (tig == 0) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        if (mt < nt) {
          part[warp * PSTRIDE + mt * 16 + gid] = acc[mt][0];
          part[warp * PSTRIDE + mt * 16 + gid + 8] = acc[mt][2];
        }
      }
    }
  }
  if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 2, ring.seq);
  if (ok) release_n(ring, ns);
  ok = consumer_sync_and<kConsumers>(ok);
  if (!ok) return false;
  float v = 0.f;
  if (t < rows) {
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) v += part[w * PSTRIDE + t];
  }
  if constexpr (SWIGLU) {
    const float up = __shfl_down_sync(0xffffffffu, v, 1);  // rows come in (gate, up) pairs
    if ((t & 1) == 0 && t < rows) out(t >> 1, v * (1.0f / (1.0f + __expf(-v))) * up);
  } else if (t < rows) {
    out(t, v);
  }
  return true;
}

// The layer's input GEMVs fused with the residual gather and RMSNorm
// (reference :121-126): warp w needs only its K slice [w K/8, (w+1) K/8) of
// the normalised input, so it polls just those residual words, writes
// bf16(h * gain) for its slice into sm.xb and runs its MMAs at once, while
// other slices may still be arriving.  The norm's scalar factor r = rsqrt(
// mean(h^2) + eps) multiplies the summed rows in the epilogue (W (h g) r
// equals W (h r g) up to where the bf16 rounding of the input falls).
// The residual comes from accumulator words (`words`, complete at `target`
// contributions; all of a lane's pending pairs are loaded before any is
// checked, so a poll costs one round trip) or, when words is null, from the
// bf16 embedding row `emb`.  keep(row, s_row, s_row+1) receives the exact
// fixed-point sums of each pair once.  Weight stages and the epilogue as
// gemv_phase_sw.
template <int K, int RB, int MT, int PSTRIDE, bool TR, bool SWIGLU, class SM, class Keep, class Out>
__device__ __forceinline__ bool gemv_x_sw(const DecodeArgs& A, RingC& ring, SM& sm, uint32_t flag, uint64_t t0,
                                          uint32_t site, const float* gain, float eps, int rows,
                                          const uint64_t* words, uint32_t target, const uint32_t* emb, Keep keep,
                                          Out out) {
  static_assert(MT * 16 <= PSTRIDE, "partial buffer");
  constexpr int KS = K / 16 / kConsumerWarps;
  constexpr int PPW = K / 2 / kConsumerWarps;  // residual pairs per warp slice
  constexpr int NPL = (PPW + 31) / 32;          // pairs per lane
  static_assert(NPL <= 32, "pending mask");
  float* part = &sm.part[0][0];
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int k0 = warp * KS * 16;
  // ---- this warp's slice of the residual -> bf16(h * gain) in sm.xb ----
  float2 g[NPL];
  uint32_t pending = 0;
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    const int p = lane + 32 * j;
    g[j] = p < PPW ? __ldg(reinterpret_cast<const float2*>(gain) + k0 / 2 + p) : make_float2(0.f, 0.f);
    if (p < PPW) pending |= 1u << j;
  }
  float hs[NPL][2];  // the lane's pairs, summed in a fixed order once all arrived
#pragma unroll
  for (int j = 0; j < NPL; ++j) hs[j][0] = hs[j][1] = 0.f;
  bool ok = true;
  Waiter wt;
  while (pending) {
    uint64_t wa[NPL], wb[NPL];
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int p = k0 / 2 + lane + 32 * j;
      if (pending & (1u << j)) {
        if (words != nullptr) {
          acc_ld2(words, p, wa[j], wb[j]);
        } else {  // embedding pair: exact bf16 values, always in the accumulator range
          const uint32_t w2 = __ldg(emb + p);
          int64_t qa = 0, qb = 0;
          acc_fix(bf16_lo(w2), qa);
          acc_fix(bf16_hi(w2), qb);
          wa[j] = (static_cast<uint64_t>(target) << kAccCountShift) + static_cast<uint64_t>(qa + target * static_cast<int64_t>(kAccBias));
          wb[j] = (static_cast<uint64_t>(target) << kAccCountShift) + static_cast<uint64_t>(qb + target * static_cast<int64_t>(kAccBias));
        }
      }
    }
#pragma unroll
    for (int j = 0; j < NPL; ++j) {
      const int p = k0 / 2 + lane + 32 * j;
      if ((pending & (1u << j)) && acc_count(wa[j]) == target && acc_count(wb[j]) == target) {
        const int64_t sa = acc_sum(wa[j], target), sb = acc_sum(wb[j], target);
        const float h0 = acc_value(sa), h1 = acc_value(sb);
        keep(2 * p, sa, sb);
        hs[j][0] = h0;
        hs[j][1] = h1;
        reinterpret_cast<__nv_bfloat162*>(sm.xb)[p] = __floats2bfloat162_rn(h0 * g[j].x, h1 * g[j].y);
        pending &= ~(1u << j);
      }
    }
    if (!pending) break;
    if (A.poll_ns) __nanosleep(A.poll_ns);
    if (wt.expired(A, flag, t0, site)) {
      ok = false;
      break;
    }
  }
  ok = __all_sync(0xffffffffu, ok);
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < NPL; ++j) {
    ss = fmaf(hs[j][0], hs[j][0], ss);
    ss = fmaf(hs[j][1], hs[j][1], ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) sm.red[warp] = ss;
  __syncwarp();  // the warp's slice of sm.xb, written by its lanes
  if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 1, ring.seq);
  // ---- the warp's K slice of every row tile ----
  const int ns = rows > 0 ? (rows + RB - 1) / RB : 0;
  ok = ok && rows <= MT * 16 && ns <= kStagesC;
  if (ok && ns > 0) ok = wait_full_n(A, ring, ns, flag, t0);
  if (ok && rows > 0) {
    const int nt = (rows + 15) >> 4;  // tiles holding rows
    const int lr = (lane & 7) + 8 * ((lane >> 3) & 1), lk = 8 * (lane >> 4);
    uint32_t rbase[MT];
    uint32_t rsw[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      const int r = min(mt * 16 + lr, rows - 1);  // rows past the range: any valid row
      const int st = r / RB, rr = r - st * RB;
      rbase[mt] = smem_addr(ring.stage[(ring.seq + static_cast<uint32_t>(st)) % kStagesC]) +
                  static_cast<uint32_t>(rr * 128);
      rsw[mt] = static_cast<uint32_t>(rr & 7);
    }
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(sm.xb);
    uint32_t bx[KS][2];
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      bx[s][0] = x32[(k0 + 16 * s + 2 * tig) >> 1];
      bx[s][1] = x32[(k0 + 16 * s + 8 + 2 * tig) >> 1];
    }
    auto a_addr = [&](int mt, int s) {
      const int kl = k0 + 16 * s + lk;
      return rbase[mt] + static_cast<uint32_t>((kl >> 6) * RB * 128) +
             ((static_cast<uint32_t>((kl >> 3) & 7) ^ rsw[mt]) << 4);
    };
    float acc[MT][4];
    uint32_t af[2][MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      acc[mt][0] = acc[mt][1] = acc[mt][2] = acc[mt][3] = 0.f;
      if (mt < nt) ldsm_x4(a_addr(mt, 0), af[0][mt][0], af[0][mt][1], af[0][mt][2], af[0][mt][3]);
    }
#pragma unroll
    for (int s = 0; s < KS; ++s) {
      if (s + 1 < KS) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
          if (mt < nt)
            ldsm_x4(a_addr(mt, s + 1), af[(s + 1) & 1][mt][0], af[(s + 1) & 1][mt][1], af[(s + 1) & 1][mt][2],
                    af[(s + 1) & 1][mt][3]);
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
        if (mt < nt)
          mma_bf16(acc[mt], af[s & 1][mt][0], af[s & 1][mt][1], af[s & 1][mt][2], af[s & 1][mt][3], bx[s][0],
                   bx[s][1]);
    }
    if (tig == 0) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        if (mt < nt) {
          part[warp * PSTRIDE + mt * 16 + gid] = acc[mt][0];
          part[warp * PSTRIDE + mt * 16 + gid + 8] = acc[mt][2];
        }
      }
    }
  }
  if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 2, ring.seq);
  if (ok) release_n(ring, ns);
  ok = consumer_sync_and<kConsumers>(ok);
  if (!ok) return false;
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < kConsumerWarps; ++w) tot += sm.red[w];
  const float r = rsqrtf(tot / static_cast<float>(K) + eps);
  float v = 0.f;
  if (t < rows) {
#pragma unroll
    for (int w = 0; w < kConsumerWarps; ++w) v += part[w * PSTRIDE + t];
    v *= r;
  }
  if constexpr (SWIGLU) {
    const float up = __shfl_down_sync(0xffffffffu, v, 1);  // rows come in (gate, up) pairs
    if ((t & 1) == 0 && t < rows) out(t >> 1, v * (1.0f / (1.0f + __expf(-v))) * up);
  } else if (t < rows) {
    out(t, v);
  }
  return true;
}

// Wo split over K: rows [0, OROWS) of this CTA's Wo boxes (row r: 64 bf16 of
// head h's columns, 128-byte swizzled) times the head output in sm.xb[0..64).
// Warp w takes 16-row tiles w, w + 8, ...; out(r, v) per row.
template <class S, class Out>
__device__ __forceinline__ bool o_phase(const DecodeArgs& A, RingC& ring, const __nv_bfloat16* xo, uint32_t flag,
                                        uint64_t t0, Out out) {
  using C = ShapeC<S>;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int gid = lane >> 2, tig = lane & 3;
  bool ok = wait_full_n(A, ring, C::OBOXES, flag, t0);
  if (ok) {
    const uint32_t* x32 = reinterpret_cast<const uint32_t*>(xo);
    for (int tile = warp; tile < C::OROWS / 16; tile += kConsumerWarps) {
      const int box = (tile * 16) / C::OBOX;
      const uint32_t sb = smem_addr(ring.stage[(ring.seq + static_cast<uint32_t>(box)) % kStagesC]);
      const int lr = tile * 16 - box * C::OBOX + (lane & 7) + 8 * ((lane >> 3) & 1);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        const int c = 2 * ks + (lane >> 4);  // 16-byte chunk of the row
        uint32_t a0, a1, a2, a3;
        ldsm_x4(sb + static_cast<uint32_t>(lr * 128 + ((c ^ (lr & 7)) << 4)), a0, a1, a2, a3);
        mma_bf16(acc, a0, a1, a2, a3, x32[8 * ks + tig], x32[8 * ks + 4 + tig]);
      }
      if (tig == 0) {
        out(tile * 16 + gid, acc[0]);
        out(tile * 16 + gid + 8, acc[2]);
      }
    }
  }
  if (ok) release_n(ring, C::OBOXES);
  return ok;
}

template <class S, bool TR>
__global__ void __launch_bounds__(kThreads, 1)
    decode_b1c_kernel(const __grid_constant__ MapsC maps, const __grid_constant__ DecodeArgs A) {
  using C = ShapeC<S>;
  extern __shared__ __align__(1024) uint8_t decode_c_smem_raw[];
  static_assert(SmemCChecks<S>::ok, "");
  const uint32_t pad = (1024u - (smem_addr(decode_c_smem_raw) & 1023u)) & 1023u;
  SmemC<S>& sm = *reinterpret_cast<SmemC<S>*>(decode_c_smem_raw + pad);
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int cta = blockIdx.x;
  const int rank = static_cast<int>(cluster_ctarank());
  const int cl = cta / kCS;
  const int head = cl < S::NH ? cl : -1;
  const int G = A.grid_part;                   // CTAs the work is split over (>= gridDim.x)
  const uint32_t n_clusters = static_cast<uint32_t>((G + kCS - 1) / kCS);
  const uint64_t t0 = globaltimer_ns();

  // No CTA returns early: one that does nothing still keeps the schedule of
  // cluster signals and the final cluster barrier (ok = false skips work).
  // A workspace holding an earlier device error stays halted until reset.
  bool ok = ld_relaxed_u32(&A.ctl->status) == 0u;
  const int nsteps = A.n_steps > 1 ? A.n_steps : 1;
  const int tok0 = A.tok ? __ldg(A.tok) : A.tok_val, pos0 = A.pos ? __ldg(A.pos) : A.pos_val;
  if (ok && (tok0 < 0 || tok0 >= A.vocab || pos0 < 0 || pos0 + nsteps > A.ctx)) {
    if (cta == 0 && t == 0)
      atomicCAS(&A.ctl->status, 0u, ST_BAD_INPUT | (tok0 < 0 || tok0 >= A.vocab ? 1u : 2u));
    ok = false;
  }
  const uint32_t flag0 = ld_relaxed_u32(&A.ctl->gen) + 1u;
  // this CTA's act chunks and logits rows (the host keeps G >= kMinGridC, so nch <= MAXCH)
  const int a8 = chunk_begin<S>(cta, G), nch = chunk_begin<S>(cta + 1, G) - a8;
  const int v0 = split_begin(cta, A.vocab, G), v1 = split_begin(cta + 1, A.vocab, G);
  ok = ok && nch <= C::MAXCH;

  if (t == 0) {
    for (int s = 0; s < kStagesC; ++s) {
      mbar_init(&sm.full[s], 1);
      mbar_init(&sm.empty[s], kConsumerWarps);
    }
    mbar_init(&sm.qkv_bar, 1);
    mbar_init(&sm.attp_bar, 1);
    mbar_init(&sm.dred_bar, 1);
    sm.abort = 0;
    fence_mbar_init();
  }
  if (warp == kConsumerWarps && lane == 0) {
    tma_prefetch_desc(&maps.qkv);
    tma_prefetch_desc(&maps.o);
    tma_prefetch_desc(&maps.gu);
    tma_prefetch_desc(&maps.down);
  }
  cluster_sync_all();  // every CTA's barriers exist before any peer signals them

  if (warp == kConsumerWarps) {
    if (ok) producer_c<S, TR>(A, sm, maps, cta, head, rank, a8, nch, v0, v1, flag0, t0, nsteps);
    return;
  }

  RingC ring{sm.stage, sm.full, sm.empty, 0u};
  uint32_t xphase = 0;  // completed phases of each cluster barrier (one per layer)
  constexpr int NP = S::NP_D;
  const int own0 = rank * C::OROWS;    // residual rows this CTA adds to the accumulators
  const bool keeper = cl == 0;         // cluster 0 carries the residual into the sums
  trace_stamp<TR>(A, 0);
  const int tf = 1 + A.n_layers * kTracePerLayer;
  for (int step = 0; step < nsteps; ++step) {
    const uint32_t flag = flag0 + static_cast<uint32_t>(step);
    const uint32_t par = flag & 1u;
    const int pos = pos0 + step;
    int tok = tok0;
    if (ok && step > 0) {  // the previous step's argmax, published by the CTA that finished it
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
      tok = sm.tok_in;
    }
    if (ok) {  // zero this CTA's share of the other parity's accumulators (the next step's)
      const size_t n2 = static_cast<size_t>(A.n_layers) * S::D * kAccStride;  // word pairs per parity
      uint4* z = reinterpret_cast<uint4*>(A.acc + static_cast<size_t>(par ^ 1u) * 2 * n2);
      const size_t za = (n2 * cta) / gridDim.x, zb = (n2 * (cta + 1)) / gridDim.x;
      for (size_t i = za + t; i < zb; i += kConsumers) z[i] = make_uint4(0u, 0u, 0u, 0u);
    }
    const int T = (pos + kCS) / kCS;  // positions per CTA: ceil((pos + 1) / kCS)
    const int p0 = min(rank * T, pos + 1), p1 = min(p0 + T, pos + 1);
    float rc = 0.f, rs = 0.f;
    if (ok && head >= 0 && t < 64) {
      rc = __ldg(A.rcos + static_cast<size_t>(pos) * 32 + (t & 31));
      rs = __ldg(A.rsin + static_cast<size_t>(pos) * 32 + (t & 31));
    }

    for (int l = 0; l < A.n_layers; ++l) {
      const int ts = 1 + l * kTracePerLayer;
      uint64_t* hm = acc_word(A, par, l, 0, S::D);
      uint64_t* hn = acc_word(A, par, l, 1, S::D);
      if (head >= 0) {
        if (ok) att_issue_c<S>(A, sm, l, head / S::GQA, pos, p0, p1);  // K/V of this layer's slice
        // ---- residual in: the embedding row (reference :87-88) or H_l; RMSNorm1;
        // q / k / v rows -> every CTA of the cluster ----
        trace_stamp<TR>(A, ts + 0);
        if (ok) {
          const uint32_t qkv_base = smem_addr(sm.qkv);
          auto push = [&](int u, float v) {
            const int comp = u / C::QROWS, idx = rank * C::QROWS + (u % C::QROWS);
            const uint32_t a = qkv_base + static_cast<uint32_t>(4 * (comp * 64 + idx));
            const uint32_t bar = smem_addr(&sm.qkv_bar);
#pragma unroll
            for (int d = 0; d < kCS; ++d) st_async_f32(mapa_shared(a, d), v, mapa_shared(bar, d));
          };
          auto keep_fix = [&](int row, int64_t sa, int64_t sb) {
            if (keeper && row >= own0 && row < own0 + C::OROWS) {
              sm.fix[row - own0] = sa;
              sm.fix[row + 1 - own0] = sb;
            }
          };
          const float* g1 = A.ln1 + static_cast<size_t>(l) * S::D;
          const uint32_t* e = reinterpret_cast<const uint32_t*>(A.wbase + A.off_emb) +
                              static_cast<size_t>(tok) * (S::D / 2);
          ok = gemv_x_sw<S::D, C::QPS, C::MT_QKV, 16 * C::MT_MAX, TR, false>(
              A, ring, sm, flag, t0, SITE_H, g1, A.eps, C::QKV_ROWS, l == 0 ? nullptr : acc_word(A, par, l - 1, 1, S::D),
              l == 0 ? 1u : n_clusters, e, keep_fix, push);
        }
        trace_stamp<TR>(A, ts + 1);
        if (ok) {
          if (t == 0) mbar_arrive_expect_tx(&sm.qkv_bar, C::kQkvBytes);
          ok = wait_cluster_bar(A, &sm.qkv_bar, xphase & 1u, flag, t0, SITE_QKVX);
        }
        ok = consumer_sync_and<kConsumers>(ok);
        trace_stamp<TR>(A, ts + 2);
        // ---- attention over this CTA's positions -> (o, m, l) to every CTA of the cluster ----
        {
          float b0 = 0.f, b1 = 0.f, M = -INFINITY, L = 0.f;
          if (ok) attention_slice<S, TR>(A, sm, l, pos, head, p0, p1, rc, rs, b0, b1, M, L, ts);
          if (ok && warp == 0) {
            const uint32_t a = smem_addr(&sm.attp[rank][2 * lane]);
            const uint32_t am = smem_addr(&sm.attp[rank][64]);
            const uint32_t bar = smem_addr(&sm.attp_bar);
#pragma unroll
            for (int d = 0; d < kCS; ++d) {
              const uint32_t rb = mapa_shared(bar, d);
              st_async_f32x2(mapa_shared(a, d), b0, b1, rb);
              if (lane == 0) st_async_f32x2(mapa_shared(am, d), M, L, rb);
            }
          }
        }
        trace_stamp<TR>(A, ts + 3);
        if (ok) {
          if (t == 0) mbar_arrive_expect_tx(&sm.attp_bar, C::kAttpBytes);
          ok = wait_cluster_bar(A, &sm.attp_bar, xphase & 1u, flag, t0, SITE_ATTX);
        }
        ok = consumer_sync_and<kConsumers>(ok);
        // ---- merge the cluster's partials (fixed order) -> head output (bf16) ----
        if (ok && t < 64) {
          float M = -INFINITY;
#pragma unroll
          for (int s = 0; s < kCS; ++s) M = fmaxf(M, sm.attp[s][64]);
          float L = 0.f, o = 0.f;
#pragma unroll
          for (int s = 0; s < kCS; ++s) {
            const float ls = sm.attp[s][65];
            const float e = ls > 0.f ? __expf(sm.attp[s][64] - M) : 0.f;
            L = fmaf(ls, e, L);
            o = fmaf(sm.attp[s][t], e, o);
          }
          sm.xb[t] = __float2bfloat16_rn(o * (1.0f / fmaxf(L, 1e-10f)));
        }
        consumer_sync<kConsumers>();
        trace_stamp<TR>(A, ts + 4);
        // ---- Wo (this CTA's rows, head h's columns) -> HM accumulators ----
        if (ok) {
          ok = o_phase<S>(A, ring, sm.xb, flag, t0, [&](int r, float v) {
            int64_t q;
            acc_contrib(A, v, keeper ? sm.fix[r] : 0, flag, SITE_HM, q);
            acc_add(hm + (own0 + r) * kAccStride, q);
          });
        }
        ok = consumer_sync_and<kConsumers>(ok);
        trace_stamp<TR>(A, ts + 5);
      }
      // ---- HM (the residual after attention); RMSNorm2; gate/up rows of this
      // CTA's act chunks -> act = silu(g) * u (bf16) ----
      trace_stamp<TR>(A, ts + 6);
      if (ok) {
        ok = gemv_x_sw<S::D, C::PS, C::MT_GU, 16 * C::MT_MAX, TR, true>(
            A, ring, sm, flag, t0, SITE_HM, A.ln2 + static_cast<size_t>(l) * S::D, A.eps, 16 * nch, hm, S::NH,
            nullptr,
            [&](int row, int64_t sa, int64_t sb) {
              if (keeper && row >= own0 && row < own0 + C::OROWS) {
                sm.fix[row - own0] = sa;
                sm.fix[row + 1 - own0] = sb;
              }
            },
            [&](int j, float a) { sm.act[j] = round_bf16(a); });
        consumer_sync<kConsumers>();
      }
      trace_stamp<TR>(A, ts + 7);
      // ---- Wd column blocks x act -> partial of every output row -> the cluster ----
      if (ok) {
        ok = wait_full_n(A, ring, nch, flag, t0);
        if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 1, ring.seq);
        if (ok) {
          // thread t: rows t + kConsumers i, independent accumulators; chunk by chunk
          constexpr int RPT = (S::D + kConsumers - 1) / kConsumers;
          float p[RPT];
#pragma unroll
          for (int i = 0; i < RPT; ++i) p[i] = 0.f;
          // (not unrolled over chunks: smaller code, measured 266.9 -> 265.1
          // us/token on config 1)
#pragma unroll 1
          for (int ch = 0; ch < nch; ++ch) {
            {
              const uint8_t* stg = ring.stage[(ring.seq + static_cast<uint32_t>(ch)) % kStagesC];
              float a[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) a[j] = sm.act[8 * ch + j];
#pragma unroll
              for (int i = 0; i < RPT; ++i) {
                const int r = t + i * kConsumers;
                if (r < S::D) {
                  const uint4 w = *reinterpret_cast<const uint4*>(stg + static_cast<size_t>(r) * 16);
                  p[i] = fmaf(a[0], bf16_lo(w.x), p[i]);
                  p[i] = fmaf(a[1], bf16_hi(w.x), p[i]);
                  p[i] = fmaf(a[2], bf16_lo(w.y), p[i]);
                  p[i] = fmaf(a[3], bf16_hi(w.y), p[i]);
                  p[i] = fmaf(a[4], bf16_lo(w.z), p[i]);
                  p[i] = fmaf(a[5], bf16_hi(w.z), p[i]);
                  p[i] = fmaf(a[6], bf16_lo(w.w), p[i]);
                  p[i] = fmaf(a[7], bf16_hi(w.w), p[i]);
                }
              }
            }
          }
#pragma unroll
          for (int i = 0; i < RPT; ++i)
            if (t + i * kConsumers < S::D) sm.u.dn.pd[t + i * kConsumers] = p[i];
          if (threadIdx.x == 0) stage_stamp<TR>(A, blockIdx.x, 2, ring.seq);
          release_n(ring, nch);
        }
        ok = consumer_sync_and<kConsumers>(ok);
        if (ok && t < S::D / 4) {  // quad t: rows 4t .. 4t + 3, owned by cluster CTA 4t / OROWS
          const int d = (4 * t) / C::OROWS;
          const float4 v = reinterpret_cast<const float4*>(sm.u.dn.pd)[t];
          st_async_f32x4(mapa_shared(smem_addr(&sm.u.dn.pr[rank][4 * t - d * C::OROWS]), d), v,
                         mapa_shared(smem_addr(&sm.dred_bar), d));
        }
      }
      trace_stamp<TR>(A, ts + 8);
      if (ok) {
        if (t == 0) mbar_arrive_expect_tx(&sm.dred_bar, C::kDredBytes);
        ok = wait_cluster_bar(A, &sm.dred_bar, xphase & 1u, flag, t0, SITE_DRED);
      }
      ok = consumer_sync_and<kConsumers>(ok);
      // ---- the cluster's sum of this CTA's rows -> H_{l+1} accumulators ----
      if (ok && t < C::OROWS) {
        float s = 0.f;
#pragma unroll
        for (int k = 0; k < kCS; ++k) s += sm.u.dn.pr[k][t];
        int64_t q;
        acc_contrib(A, s, keeper ? sm.fix[t] : 0, flag, SITE_H, q);
        acc_add(hn + (own0 + t) * kAccStride, q);
      }
      trace_stamp<TR>(A, ts + 9);
      ++xphase;
      if (head >= 0) consumer_sync<kConsumers>();  // down partials read before the next layer's K/V copies
    }

    // ---- final norm + tied logits + argmax (reference :314-357) ----
    {
      float2 g[NP];
      load_gain_pairs<S, NP>(A.lnf, g);
      float hv[NP][2];
#pragma unroll
      for (int i = 0; i < NP; ++i) hv[i][0] = hv[i][1] = 0.f;
      bool got = ok;
      if (ok)
        got = gather_acc<S, NP>(A, acc_word(A, par, A.n_layers - 1, 1, S::D), n_clusters, flag, t0, SITE_FINAL, hv,
                                [](int, int64_t, int64_t) {});
      ok = norm_x<S, NP>(sm, hv, g, A.eps, got) && ok;
    }
    trace_stamp<TR>(A, tf + 0);
    if (ok) {
      const XSmem x{reinterpret_cast<const uint4*>(sm.xb)};
      float best_v = -INFINITY;
      int best_i = 0x7fffffff;
      // released two stages at a time, so up to 10 of the 12 slots can be in flight
      ok = gemv_phase_wide<S::KD, S::ROWB_D, S::RPS_D, RingC, 2, TR>(A, ring, flag, t0, v0, v1, x, [&](int u, float v, float) {
        if (lane == 0 && A.logits) A.logits[u] = v;
        if (v > best_v) {
          best_v = v;
          best_i = u;
        }
      });
      ok = consumer_sync_and<kConsumers>(ok);
      trace_stamp<TR>(A, tf + 1);
      if (ok) {
        if (lane == 0) {
          sm.am_v[warp] = best_v;
          sm.am_i[warp] = best_i;
        }
        consumer_sync<kConsumers>();
        if (t == 0) {
          float bv = sm.am_v[0];
          int bi = sm.am_i[0];
          for (int w = 1; w < kConsumerWarps; ++w) {
            if (sm.am_v[w] > bv || (sm.am_v[w] == bv && sm.am_i[w] < bi)) {
              bv = sm.am_v[w];
              bi = sm.am_i[w];
            }
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
              if (v > gv || (v == gv && i < gi)) {
                gv = v;
                gi = i;
              }
            }
            const int tk = gi == 0x7fffffff ? 0 : gi;
            *A.next_tok = tk;
            if (A.tok_out != nullptr) A.tok_out[step] = tk;
            A.ctl->arrive = 0u;
            __threadfence();
            st_relaxed_u32(&A.ctl->gen, flag);
            if (step + 1 < nsteps)
              st_release_u64(&A.ctl->tok_word, (static_cast<uint64_t>(flag) << 32) | static_cast<uint32_t>(tk));
          }
        }
      }
    }
  }  // step
  trace_stamp<TR>(A, tf + 2);
  if (!ok) *reinterpret_cast<volatile int*>(&sm.abort) = 1;
  cp_async_wait_all();  // K/V copies of a layer whose attention was skipped
  __syncwarp();
  // No CTA leaves while a peer may still store into its shared memory or
  // arrive on its barriers (all pushes precede every CTA's arrival here).
  cluster_sync_all();
}

}  // namespace b2d
