// sampler.cuh — device sampler: one CTA per sequence, or for top-p draws a
// cluster of 16 or 8 CTAs per sequence while the batch fits one wave (sm_100a).
//
// Replaces the reference's host numpy sampler, generate.py:28-65 sample_token:
// repetition penalty over the set of generated tokens, temperature, softmax,
// top-p (nucleus) filtering, and numpy's legacy RandomState.choice, which
// draws one uniform u and returns keep[searchsorted(cumsum(p64)/last, u,
// 'right')].  The caller supplies u (float64), so a token is a function of
// (logits, u) alone.  The arithmetic follows the reference's order so the token
// equals the CPU restatement's:
//   * penalty / temperature: float32 IEEE division or product by the
//     float32-rounded parameter (numpy's weak Python-float scalars);
//   * exp: the float64 exponential rounded to float32 (host independent; the
//     reference's own np.exp is host dependent, up to 2 ulp on AVX-512);
//   * normalisers: numpy's pairwise float32 summation (blocks of <= 128 with 8
//     accumulators, halving at multiples of 8), evaluated as a tree;
//   * top-p: order by descending probability, ties by ascending token id (a
//     stable radix sort of the probabilities, which start in id order); the
//     cutoff from a sequential float32 cumsum compared in float64 (numpy's
//     searchsorted promotes the Python float);
//   * choice: float64 prefix sums, divided by the total, first value > u.  The
//     prefix sums are computed in parallel, so their last bits can differ from
//     numpy's sequential cumsum; a token differs only if u falls within about
//     1e-12 of a CDF boundary.
// Everything for one sequence lives in shared memory (vocabularies up to
// kSamplerMaxVocab); nothing is allocated.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "b2d_ptx.cuh"
#include "tc_ptx.cuh"

namespace b2d {

constexpr int kSamplerMaxVocab = 32768;
constexpr int kSamplerThreads = 1024;
constexpr int kTreeNodes = 1024;  // heap-indexed pairwise-sum tree (depth <= 9)
// Cluster sampler: one cluster of CL (8 or 16) CTAs per sequence, CTA r
// holding sort positions [r * slice, (r + 1) * slice), slice =
// kSamplerMaxVocab / CL.
constexpr int kSampleCluster = 8;      // the portable cluster size
constexpr int kSampleClusterMax = 16;  // where the device runs clusters of 16
static_assert(kSamplerMaxVocab / kSampleClusterMax >= kSamplerThreads, "at least one position per thread");

struct SampleArgs {
  const float* logits;     // [batch][vocab]
  const int32_t* history;  // [batch][hist_cap] or null
  const int32_t* hist_len; // [batch] or null
  const double* uniforms;  // [batch] or null (temperature == 0)
  int32_t* out;            // [batch]
  int vocab, hist_cap;
  float temperature, rep_penalty;
  double top_p;
  uint64_t* trace;         // diagnostics: global-timer stamps [batch][8] (thread 0 of each CTA), or null
  uint64_t* scratch;       // [batch][kSamplerMaxVocab] radix-sort buffer (key << 32 | id)
};

struct SamplerSmem {
  uint32_t key[kSamplerMaxVocab];   // float bits of p, then ~bits for the sort
  uint16_t idx[kSamplerMaxVocab];   // token id travelling with the key
  uint32_t seen[kSamplerMaxVocab / 32];
  int node_start[kTreeNodes];
  int node_len[kTreeNodes];
  float node_val[kTreeNodes];
  double red_d[kSamplerThreads / 32];
  float red_f[kSamplerThreads / 32];
  int red_i[kSamplerThreads / 32];
  int cutoff;
  int token;
  // top-p cutoff state: the exact float32 running sum c of the sorted
  // probabilities before element ch_k, the result (0 = not found yet), and the
  // first event of a parallel round (position, prefix before it, kind)
  float ch_c;
  int ch_k, ch_cut, ev_k, ev_kind;
  long long ev_s, ch_tot;
  long long scan64[kSamplerThreads / 32];
  int rs_cnt[kSamplerThreads / 32][17];  // radix sort: digit counts / running offsets per warp
  int rs_off[kSamplerThreads / 32][17];  // (rows padded: a column read is conflict-free)
  // cluster sampler: values every CTA of the cluster pushes into every CTA
  // (slot = the pushing CTA's rank)
  float cl_max[kSampleClusterMax];
  uint32_t cl_and[kSampleClusterMax], cl_or[kSampleClusterMax];
  int cl_cnt[kSampleClusterMax][16];
  int cl_tot[16], cl_lstart[16], cl_gofs[16];  // a sort pass's digit totals and starts: in the stage, stage -> global
  uint32_t red_and[kSamplerThreads / 32], red_or[kSamplerThreads / 32];
};

__device__ __forceinline__ float key_to_p(uint32_t k) { return __uint_as_float(~k); }

// numpy's pairwise float32 sum, evaluated as a heap-indexed tree of its
// recursion: every node longer than 128 splits at n2 = n/2 rounded down to a
// multiple of 8; a leaf (<= 128) is numpy's 8-accumulator block sum.
// tree_split builds the nodes of the range [0, n) (all threads of the block).
__device__ void tree_split(SamplerSmem& sm, int n) {
  const int t = threadIdx.x;
  for (int i = t; i < kTreeNodes; i += blockDim.x) sm.node_len[i] = -1;
  __syncthreads();
  if (t == 0) {
    sm.node_start[1] = 0;
    sm.node_len[1] = n;
  }
  __syncthreads();
  for (int d = 0; d < 9; ++d) {
    const int first = 1 << d, count = 1 << d;
    for (int i = t; i < count; i += blockDim.x) {
      const int nd = first + i;
      const int len = sm.node_len[nd];
      if (len > 128 && 2 * nd + 1 < kTreeNodes) {
        int n2 = len / 2;
        n2 -= n2 % 8;
        sm.node_start[2 * nd] = sm.node_start[nd];
        sm.node_len[2 * nd] = n2;
        sm.node_start[2 * nd + 1] = sm.node_start[nd] + n2;
        sm.node_len[2 * nd + 1] = len - n2;
      }
    }
    __syncthreads();
  }
}

// Bottom-up: internal node = left + right; returns 0 + root like np.sum.
__device__ float tree_combine(SamplerSmem& sm) {
  const int t = threadIdx.x;
  for (int d = 8; d >= 0; --d) {
    const int first = 1 << d, count = 1 << d;
    for (int i = t; i < count; i += blockDim.x) {
      const int nd = first + i;
      if (sm.node_len[nd] > 128 && 2 * nd + 1 < kTreeNodes)
        sm.node_val[nd] = __fadd_rn(sm.node_val[2 * nd], sm.node_val[2 * nd + 1]);
    }
    __syncthreads();
  }
  const float total = __fadd_rn(0.f, sm.node_val[1]);
  __syncthreads();
  return total;
}

// The leaves of the split tree, eight lanes per leaf (four leaves per warp):
// lane j of a leaf's group runs numpy's accumulator j over elements
// s0 + 8i + j, so the group reads 8 consecutive words per step (one thread
// per leaf would read words 8 apart: 8-way bank conflicts).  The group then
// adds ((r0 + r1) + (r2 + r3)) + ((r4 + r5) + (r6 + r7)) by shuffles and its
// first lane the remainder, numpy's order exactly.  `mine(s0)` says whether
// this CTA computes the leaf starting at s0; `store(nd, v)` (first lane of the
// group) receives each leaf's sum.  Every warp of the block must call it.
template <class Get, class Mine, class Store>
__device__ void tree_leaves(const SamplerSmem& sm, Get get, Mine mine, Store store) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, j = lane & 7;
  const int nwarps = static_cast<int>(blockDim.x) >> 5;
  for (int base = 4 * warp; base < kTreeNodes; base += 4 * nwarps) {
    const int nd = base + (lane >> 3);
    const int len = sm.node_len[nd], s0 = sm.node_start[nd];
    const bool leaf = len >= 0 && len <= 128 && mine(s0);
    if (!__any_sync(0xffffffffu, leaf)) continue;
    const int body = len - (len % 8);
    float r = 0.f;
    if (leaf && len >= 8) {
      r = get(s0 + j);
      for (int i = 8; i < body; i += 8) r = __fadd_rn(r, get(s0 + i + j));
    }
    r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 1));
    r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 2));
    r = __fadd_rn(r, __shfl_xor_sync(0xffffffffu, r, 4));
    if (leaf && j == 0) {
      float res;
      if (len < 8) {
        res = 0.f;
        for (int i = 0; i < len; ++i) res = __fadd_rn(res, get(s0 + i));
      } else {
        res = r;
        for (int i = body; i < len; ++i) res = __fadd_rn(res, get(s0 + i));
      }
      store(nd, res);
    }
  }
}

// numpy's pairwise float32 sum of get(0..n-1) (n <= 2^16, so the tree's leaves
// are at most 128 long); all threads of the block must call it.
template <class Get>
__device__ float pairwise_sum(SamplerSmem& sm, int n, Get get) {
  tree_split(sm, n);
  tree_leaves(sm, get, [](int) { return true; }, [&](int nd, float v) { sm.node_val[nd] = v; });
  __syncthreads();
  return tree_combine(sm);
}

// Block-wide float64 prefix sums of get(0..n-1) (thread-contiguous chunks);
// returns the first k with prefix_k / total > u (numpy's searchsorted 'right'
// after cdf /= cdf[-1]).
template <class Get>
__device__ int cdf_search(SamplerSmem& sm, int n, double u, Get get) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  // thread-contiguous chunks of an odd length: lanes' reads then fall in
  // distinct banks (an even length such as 28 conflicts 4- to 8-way)
  const int per = ((n + kSamplerThreads - 1) / kSamplerThreads) | 1;
  const int i0 = min(t * per, n), i1 = min(i0 + per, n);
  double local = 0.0;
  for (int i = i0; i < i1; ++i) local += static_cast<double>(get(i));
  // exclusive scan of the thread sums
  double incl = local;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const double v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) sm.red_d[warp] = incl;
  __syncthreads();
  constexpr int kWarps = kSamplerThreads / 32;
  if (warp == 0) {
    double w = lane < kWarps ? sm.red_d[lane] : 0.0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double v = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += v;
    }
    if (lane < kWarps) sm.red_d[lane] = w;  // inclusive warp-total prefix
  }
  __syncthreads();
  const double total = sm.red_d[kWarps - 1];
  const double run0 = (warp > 0 ? sm.red_d[warp - 1] : 0.0) + (incl - local);
  // The running sums never decrease and a correctly rounded division is
  // monotone in its dividend, so only the chunk whose end already exceeds u
  // can hold the first crossing: one division per chunk, then per element
  // in that chunk alone.
  double run = run0;
  for (int i = i0; i < i1; ++i) run += static_cast<double>(get(i));
  int found = 0x7fffffff;
  if (i1 > i0 && run / total > u) {
    run = run0;
    for (int i = i0; i < i1; ++i) {
      run += static_cast<double>(get(i));
      if (run / total > u) { found = i; break; }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) found = min(found, __shfl_xor_sync(0xffffffffu, found, o));
  __syncthreads();
  if (lane == 0) sm.red_i[warp] = found;
  __syncthreads();
  int k = 0x7fffffff;
  for (int w = 0; w < kSamplerThreads / 32; ++w) k = min(k, sm.red_i[w]);
  __syncthreads();
  return k == 0x7fffffff ? n - 1 : k;
}

// Lanes of the warp whose 4-bit digit equals this lane's.
__device__ __forceinline__ uint32_t same_digit_lanes(uint32_t d) {
  uint32_t m = 0xffffffffu;
#pragma unroll
  for (int bit = 0; bit < 4; ++bit) {
    const uint32_t bal = __ballot_sync(0xffffffffu, (d >> bit) & 1u);
    m &= ((d >> bit) & 1u) ? bal : ~bal;
  }
  return m;
}

// Stable LSD radix sort of (key, id) ascending by key: 8 passes of 4 bits,
// alternating shared memory (sm.key / sm.idx) and the sequence's global
// scratch (key << 32 | id); the result ends in shared memory.  Warp w owns
// elements [1024 w, 1024 w + 1024) and visits them in index order (32 rounds
// of 32 consecutive elements), so equal keys keep their order: the initial
// order is by token id, hence ties end ascending by id, the order of the
// (-p, id) comparison.  All threads of the block must call it.
__device__ void radix_sort(SamplerSmem& sm, uint64_t* gbuf) {
  static_assert(kSamplerMaxVocab == 32 * kSamplerThreads, "one 1024-element block per warp");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t below = (1u << lane) - 1u;
  for (int pass = 0; pass < 8; ++pass) {
    const int sh = 4 * pass;
    const bool src_smem = (pass & 1) == 0;
    if (lane < 16) sm.rs_cnt[warp][lane] = 0;
    __syncwarp();
#pragma unroll 4
    for (int r = 0; r < 32; ++r) {  // digit counts of this warp's block
      const int i = warp * 1024 + r * 32 + lane;
      const uint32_t k = src_smem ? sm.key[i] : static_cast<uint32_t>(__ldcg(gbuf + i) >> 32);
      atomicAdd(&sm.rs_cnt[warp][(k >> sh) & 15u], 1);
    }
    __syncthreads();
    if (warp == 0) {  // offsets: digit d's elements of warp w start at base(d) + sum over earlier warps
      int tot = 0;
      if (lane < 16)
        for (int w = 0; w < kSamplerThreads / 32; ++w) {
          const int c = sm.rs_cnt[w][lane];
          sm.rs_off[w][lane] = tot;
          tot += c;
        }
      int incl = tot;
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += v;
      }
      if (lane < 16)
        for (int w = 0; w < kSamplerThreads / 32; ++w) sm.rs_off[w][lane] += incl - tot;
    }
    __syncthreads();
#pragma unroll 2
    for (int r = 0; r < 32; ++r) {  // scatter in index order
      const int i = warp * 1024 + r * 32 + lane;
      uint32_t k, x;
      if (src_smem) {
        k = sm.key[i];
        x = sm.idx[i];
      } else {
        const uint64_t v = __ldcg(gbuf + i);
        k = static_cast<uint32_t>(v >> 32);
        x = static_cast<uint32_t>(v) & 0xffffu;
      }
      const uint32_t d = (k >> sh) & 15u;
      const uint32_t m = same_digit_lanes(d);
      const int dst = sm.rs_off[warp][d] + __popc(m & below);
      __syncwarp();
      if ((m & below) == 0) sm.rs_off[warp][d] += __popc(m);  // the group's lowest lane advances it
      __syncwarp();
      if (src_smem) {
        __stcg(gbuf + dst, (static_cast<uint64_t>(k) << 32) | x);
      } else {
        sm.key[dst] = k;
        sm.idx[dst] = static_cast<uint16_t>(x);
      }
    }
    __syncthreads();  // the pass's output is complete (global and shared) before the next pass reads it
  }
}

// numpy's top-p cutoff on the sorted probabilities p_k = key_to_p(key[k]):
// the first k + 1 with float64(c_k) >= top_p, where c_k = fl32(c_{k-1} + p_k)
// is numpy's sequential float32 cumsum (V if never).  float64(c) >= top_p is
// c >= thr with thr = top_p rounded up to a float.
//
// The chain is evaluated exactly but in parallel.  While the running sum c
// stays in one binade [2^E, 2^(E+1)) it is an integer multiple of u = 2^(E-23),
// and fl32(c + p) = c + u * round(p / u) (round to nearest) unless p / u has a
// fractional part of exactly 1/2 (then the tie goes to the even multiple,
// which depends on c).  So a round of the block scales a chunk of 8 elements
// per thread by 1/u, takes the integer prefix sums of the rounded values, and
// finds the first element that (a) is a tie, (b) would carry the sum into the
// next binade, or (c) reaches thr.  Events (a) and (b) are resolved with one
// ordinary float32 addition and the next round starts after them; (c) ends.
// The first kSeqHead elements, where c is small and changes binade often,
// run sequentially (in blocks of 16 prefetched keys).  Sorted descending, every later p_k <= c, so p / u < 2^24.
__device__ int topp_cutoff(SamplerSmem& sm, int V, double top_p, uint64_t* diag, int& rounds) {
  constexpr int kSeqHead = 512, kPer = 8, kChunk = kPer * kSamplerThreads;
  constexpr int kWarps = kSamplerThreads / 32;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float thr = __double2float_ru(top_p);
  if (t == 0) {  // the head, 16 keys per block: the sum never decreases, so a
                 // block whose end stays below thr needs no per-key test
    const uint4* k4 = reinterpret_cast<const uint4*>(sm.key);
    const int n0 = min(kSeqHead, V);  // a multiple of 16, or V
    float c = 0.f;
    int cut = 0, base = 0;
    uint4 nxt[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) nxt[q] = k4[q];
    for (; base < n0; base += 16) {
      uint4 cur[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) cur[q] = nxt[q];
#pragma unroll
      for (int q = 0; q < 4; ++q) nxt[q] = base + 16 + 4 * q < kSamplerMaxVocab ? k4[(base + 16) / 4 + q] : cur[q];
      float e = c;
      const int nk = min(16, n0 - base);
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // keys at or past V decode to p = 0
        e = __fadd_rn(e, 4 * q + 0 < nk ? key_to_p(cur[q].x) : 0.f);
        e = __fadd_rn(e, 4 * q + 1 < nk ? key_to_p(cur[q].y) : 0.f);
        e = __fadd_rn(e, 4 * q + 2 < nk ? key_to_p(cur[q].z) : 0.f);
        e = __fadd_rn(e, 4 * q + 3 < nk ? key_to_p(cur[q].w) : 0.f);
      }
      if (e >= thr) {
        for (int i = 0; i < nk; ++i) {
          c = __fadd_rn(c, key_to_p(sm.key[base + i]));
          if (c >= thr) {
            cut = base + i + 1;
            break;
          }
        }
        break;
      }
      c = e;
    }
    sm.ch_c = c;
    sm.ch_k = cut ? cut : n0;
    sm.ch_cut = cut ? cut : (n0 == V ? V : 0);
    if (diag) diag[0] = globaltimer_ns();
  }
  __syncthreads();
  rounds = 0;
  constexpr uint32_t kSat = 1u << 30;  // scans saturate here: any sum that large is past an event
  while (sm.ch_cut == 0) {
    ++rounds;
    const int k0 = sm.ch_k;
    const int k0a = k0 & ~(kPer - 1);  // the chunk starts 8-aligned; keys before k0 count as p = 0
    const float c = sm.ch_c;  // > 0: it holds p_0, the largest probability
    int ex;
    frexpf(c, &ex);  // c in [2^(ex-1), 2^ex): ulp u = 2^(ex-24)
    const float scale = ldexpf(1.0f, 24 - ex);  // 1 / u, a power of two
    const uint32_t c0 = static_cast<uint32_t>(__fmul_rn(c, scale));  // c / u, exact (< 2^24)
    // T: the first running sum (in units of u) that reaches thr
    const double Td = ceil(static_cast<double>(thr) * static_cast<double>(scale));
    const uint32_t T = Td >= 2147483648.0 ? 0x80000000u : static_cast<uint32_t>(Td);
    const int kb = k0a + kPer * t;
    uint32_t kw[kPer];
    if (kb < kSamplerMaxVocab) {  // two 16-byte loads: 2-way bank conflicts instead of 8-way
      const uint4 lo = *reinterpret_cast<const uint4*>(&sm.key[kb]);
      const uint4 hi = *reinterpret_cast<const uint4*>(&sm.key[kb + 4]);
      kw[0] = lo.x; kw[1] = lo.y; kw[2] = lo.z; kw[3] = lo.w;
      kw[4] = hi.x; kw[5] = hi.y; kw[6] = hi.z; kw[7] = hi.w;
    } else {
#pragma unroll
      for (int j = 0; j < kPer; ++j) kw[j] = 0xffffffffu;
    }
    float y[kPer];
    uint32_t loc = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int k = kb + j;
      const float p = (k >= k0 && k < V) ? key_to_p(kw[j]) : 0.f;
      y[j] = __fmul_rn(p, scale);  // p / u, exact, < 2^24
      const float q = floorf(y[j]);
      loc += static_cast<uint32_t>(q) + (y[j] - q > 0.5f ? 1u : 0u);
    }
    // block scan of the per-thread sums (32-bit, saturating)
    uint32_t inc = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc = min(inc + v, kSat);
    }
    const uint32_t excl = __shfl_up_sync(0xffffffffu, inc, 1);
    if (lane == 31) sm.scan64[warp] = inc;
    if (t == 0) sm.ev_k = 0x7fffffff;
    __syncthreads();
    uint32_t wt = lane < kWarps ? static_cast<uint32_t>(sm.scan64[lane]) : 0u;  // every warp scans the warp totals
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t v = __shfl_up_sync(0xffffffffu, wt, o);
      if (lane >= o) wt = min(wt + v, kSat);
    }
    const uint32_t wbefore = __shfl_sync(0xffffffffu, wt, (warp + 31) & 31);
    uint32_t S = min(c0 + (warp > 0 ? wbefore : 0u) + (lane > 0 ? excl : 0u), kSat);
    int ev = 0x7fffffff, kind = 0;
    uint32_t ev_s = 0;
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const int k = kb + j;
      if (k < k0 || k >= V || ev != 0x7fffffff) continue;
      const float q = floorf(y[j]);
      const float f = y[j] - q;
      const uint32_t qi = static_cast<uint32_t>(q);
      if (f == 0.5f || S + qi >= (1u << 24) - 2) {  // exact tie, or the sum may leave the binade
        ev = k; kind = 1; ev_s = S;
        continue;
      }
      S += qi + (f > 0.5f ? 1u : 0u);
      if (S >= T) {  // threshold reached at k
        ev = k; kind = 2; ev_s = S;
      }
    }
    if (ev != 0x7fffffff) atomicMin(&sm.ev_k, ev);
    __syncthreads();
    if (ev != 0x7fffffff && ev == sm.ev_k) {  // the owner of the first event
      sm.ev_kind = kind;
      sm.ev_s = ev_s;
    }
    if (t == kSamplerThreads - 1) sm.ch_tot = S;  // the chunk's end (used when no event)
    __syncthreads();
    if (t == 0) {
      const int k = sm.ev_k;
      const float u = ldexpf(1.0f, ex - 24);
      if (k == 0x7fffffff) {  // no event: the whole chunk stays in the binade, below thr
        const int end = min(k0a + kChunk, V);
        sm.ch_c = __fmul_rn(static_cast<float>(sm.ch_tot), u);  // < 2^24 units: exact
        sm.ch_k = end;
        if (end >= V) sm.ch_cut = V;
      } else if (sm.ev_kind == 2) {
        sm.ch_cut = k + 1;
      } else {
        const float cb = __fmul_rn(static_cast<float>(sm.ev_s), u);  // the exact sum before k
        const float ck = __fadd_rn(cb, key_to_p(sm.key[k]));
        if (ck >= thr) {
          sm.ch_cut = k + 1;
        } else {
          sm.ch_c = ck;
          sm.ch_k = k + 1;
          if (k + 1 >= V) sm.ch_cut = V;
        }
      }
    }
    __syncthreads();
  }
  const int cut = sm.ch_cut;
  __syncthreads();
  return cut;
}

__global__ void __launch_bounds__(kSamplerThreads, 1) sample_kernel(const SampleArgs a) {
  extern __shared__ __align__(16) uint8_t sampler_smem_raw[];
  SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(sampler_smem_raw);
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int V = a.vocab;
  const float* lg = a.logits + static_cast<size_t>(b) * V;
  constexpr int PER = kSamplerMaxVocab / kSamplerThreads;
  // stamps: 0 entry, 1 exponentials, 2 normalised, 3 sorted, 4 cutoff, 5 drawn;
  // slot 6 = the top-p cutoff (tokens kept) | parallel rounds of the cutoff << 32,
  // slot 7 = end of the cutoff's sequential head (global timer)
  auto stamp = [&](int slot) {
    if (a.trace != nullptr && t == 0) a.trace[static_cast<size_t>(b) * 8 + slot] = globaltimer_ns();
  };
  stamp(0);

  // ---- repetition penalty over the set of generated tokens (ref :32-39) ----
  const int hl = (a.history && a.hist_len) ? min(max(a.hist_len[b], 0), a.hist_cap) : 0;
  const bool penalize = a.rep_penalty != 1.0f && hl > 0;
  if (penalize) {
    for (int i = t; i < kSamplerMaxVocab / 32; i += kSamplerThreads) sm.seen[i] = 0u;
    __syncthreads();
    for (int i = t; i < hl; i += kSamplerThreads) {
      const int tok = a.history[static_cast<size_t>(b) * a.hist_cap + i];
      if (tok >= 0 && tok < V) atomicOr(&sm.seen[tok >> 5], 1u << (tok & 31));
    }
    __syncthreads();
  }
  float v[PER];
#pragma unroll
  for (int r = 0; r < PER; ++r) {
    const int i = t + r * kSamplerThreads;
    float x = -INFINITY;
    if (i < V) {
      x = lg[i];
      if (penalize && (sm.seen[i >> 5] >> (i & 31)) & 1u)
        x = x > 0.f ? __fdiv_rn(x, a.rep_penalty) : __fmul_rn(x, a.rep_penalty);
    }
    v[r] = x;
  }

  // ---- greedy: first index of the maximum (ref :41-42, np.argmax) ----
  if (a.temperature == 0.0f) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int r = 0; r < PER; ++r) {
      const int i = t + r * kSamplerThreads;
      if (i < V && (v[r] > bv || (v[r] == bv && i < bi))) { bv = v[r]; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { sm.red_f[warp] = bv; sm.red_i[warp] = bi; }
    __syncthreads();
    if (t == 0) {
      float gv = sm.red_f[0];
      int gi = sm.red_i[0];
      for (int w = 1; w < kSamplerThreads / 32; ++w)
        if (sm.red_f[w] > gv || (sm.red_f[w] == gv && sm.red_i[w] < gi)) { gv = sm.red_f[w]; gi = sm.red_i[w]; }
      a.out[b] = gi == 0x7fffffff ? 0 : gi;
    }
    return;
  }

  // ---- temperature, max shift, exp (ref :44-50) ----
  float mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < PER; ++r) {
    if (a.temperature != 1.0f && t + r * kSamplerThreads < V) v[r] = __fdiv_rn(v[r], a.temperature);
    mx = fmaxf(mx, v[r]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) sm.red_f[warp] = mx;
  __syncthreads();
  mx = sm.red_f[0];
  for (int w = 1; w < kSamplerThreads / 32; ++w) mx = fmaxf(mx, sm.red_f[w]);
#pragma unroll
  for (int r = 0; r < PER; ++r) {
    const int i = t + r * kSamplerThreads;
    if (i < V) {
      const float sh = __fsub_rn(v[r], mx);
      sm.key[i] = __float_as_uint(__double2float_rn(exp(static_cast<double>(sh))));
    }
  }
  __syncthreads();
  stamp(1);
  // ---- normalise: p /= p.sum() (ref :51) ----
  const float S = pairwise_sum(sm, V, [&](int i) { return __uint_as_float(sm.key[i]); });
  const bool top = a.top_p < 1.0;
  for (int i = t; i < kSamplerMaxVocab; i += kSamplerThreads) {
    if (i < V) {
      const float p = __fdiv_rn(__uint_as_float(sm.key[i]), S);
      sm.key[i] = top ? ~__float_as_uint(p) : __float_as_uint(p);
    } else {
      sm.key[i] = 0xffffffffu;  // sorts after every real key
    }
    sm.idx[i] = static_cast<uint16_t>(i < V ? i : 0xffff);
  }
  __syncthreads();

  if (!top) {  // choice over all tokens in id order (ref :65)
    const int k = cdf_search(sm, V, a.uniforms[b], [&](int i) { return __uint_as_float(sm.key[i]); });
    if (t == 0) a.out[b] = k;
    return;
  }

  // ---- top-p (ref :53-63): sort by (descending p, ascending id) ----
  // key = ~bits of p: ascending keys are descending probabilities.
  stamp(2);
  radix_sort(sm, a.scratch + static_cast<size_t>(b) * kSamplerMaxVocab);
  stamp(3);
  int n_rounds = 0;
  const int cut = topp_cutoff(sm, V, a.top_p, a.trace != nullptr ? a.trace + static_cast<size_t>(b) * 8 + 7 : nullptr, n_rounds);
  if (a.trace != nullptr && t == 0)
    a.trace[static_cast<size_t>(b) * 8 + 6] = static_cast<uint64_t>(cut) | (static_cast<uint64_t>(n_rounds) << 32);
  stamp(4);
  const float S2 = pairwise_sum(sm, cut, [&](int i) { return key_to_p(sm.key[i]); });
  for (int i = t; i < cut; i += kSamplerThreads)  // the renormalised kept p, once each
    sm.key[i] = __float_as_uint(__fdiv_rn(key_to_p(sm.key[i]), S2));
  __syncthreads();
  const int k = cdf_search(sm, cut, a.uniforms[b], [&](int i) { return __uint_as_float(sm.key[i]); });
  if (t == 0) a.out[b] = sm.idx[k];
  stamp(5);
}

// The top-p sampler on a cluster of kSampleCluster CTAs per sequence
// (temperature > 0, top_p < 1).  Same arithmetic, and so the same token, as
// sample_kernel; the work that scales with the vocabulary is spread over the
// cluster:
//   * CTA r takes token ids [r * kSliceElems, (r + 1) * kSliceElems):
//     penalty, temperature, its max (exchanged), float64 exp;
//   * the pairwise sum's leaves are summed where they start (reading a
//     neighbour's exponentials through distributed shared memory where a leaf
//     crosses a slice), broadcast to every CTA, and combined identically in
//     each;
//   * the stable LSD radix sort (4-bit digits) keeps sort positions [r *
//     kSliceElems, ...) in CTA r: each pass counts digits per warp, exchanges
//     the CTA's 16 totals, orders its elements by digit in a local stage, and
//     sends each digit's run to its consecutive destination positions (in
//     whichever CTAs hold them).  (4096 random 8-byte stores into other
//     CTAs took ~5,900 cycles per CTA, ~900 into its own shared memory.)  Digits that are equal for every
//     key (from the keys' AND / OR, exchanged with the first pass's counts)
//     are skipped: such a pass is the identity;
//   * the sorted keys and ids are gathered into CTA 0, which runs the top-p
//     cutoff, the renormalisation and the draw alone.
// Every thread of every CTA passes every cluster barrier (no early exit
// before the gather), and no wait depends on data.  Before the gather, CTA
// r's shared key array holds two sort buffers and its exponentials.
template <int SLICE>
__device__ __forceinline__ uint64_t* cl_sort_buf(SamplerSmem& sm, int which) {
  return reinterpret_cast<uint64_t*>(sm.key) + which * SLICE;
}
template <int SLICE>
__device__ __forceinline__ float* cl_exp_buf(SamplerSmem& sm) {
  return reinterpret_cast<float*>(sm.key + 4 * SLICE);
}

template <int CL>
__global__ void __launch_bounds__(kSamplerThreads, 1) sample_cluster_kernel(const SampleArgs a) {
  constexpr int kSliceElems = kSamplerMaxVocab / CL;       // positions per CTA
  constexpr int PT = kSliceElems / kSamplerThreads;        // per thread
  constexpr int WPOS = kSliceElems / (kSamplerThreads / 32);  // per warp
  static_assert(PT * kSamplerThreads == kSliceElems && CL <= 16, "slice layout");
  extern __shared__ __align__(16) uint8_t sampler_smem_raw[];
  SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(sampler_smem_raw);
  const int rank = static_cast<int>(cluster_ctarank());
  const int b = blockIdx.x / CL, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int V = a.vocab;
  const int i0 = rank * kSliceElems;
  const int nloc = max(0, min(kSliceElems, V - i0));  // positions (and ids) this CTA holds
  const float* lg = a.logits + static_cast<size_t>(b) * V;
  const bool lead = rank == 0;
  constexpr int kWarps = kSamplerThreads / 32;
  auto stamp = [&](int slot) {
    if (a.trace != nullptr && lead && t == 0) a.trace[static_cast<size_t>(b) * 8 + slot] = globaltimer_ns();
  };
  cluster_sync_all();  // every CTA of the cluster runs before any writes into another
  stamp(0);

  // ---- penalty, temperature, max (ref :32-49) ----
  const int hl = (a.history && a.hist_len) ? min(max(a.hist_len[b], 0), a.hist_cap) : 0;
  const bool penalize = a.rep_penalty != 1.0f && hl > 0;
  if (penalize) {
    for (int i = t; i < kSliceElems / 32; i += kSamplerThreads) sm.seen[i] = 0u;
    __syncthreads();
    for (int i = t; i < hl; i += kSamplerThreads) {
      const int tok = a.history[static_cast<size_t>(b) * a.hist_cap + i] - i0;
      if (tok >= 0 && tok < nloc) atomicOr(&sm.seen[tok >> 5], 1u << (tok & 31));
    }
    __syncthreads();
  }
  float v[PT];
  float mx = -INFINITY;
#pragma unroll
  for (int r = 0; r < PT; ++r) {
    const int j = t + r * kSamplerThreads;
    float x = -INFINITY;
    if (j < nloc) {
      x = lg[i0 + j];
      if (penalize && (sm.seen[j >> 5] >> (j & 31)) & 1u)
        x = x > 0.f ? __fdiv_rn(x, a.rep_penalty) : __fmul_rn(x, a.rep_penalty);
      if (a.temperature != 1.0f) x = __fdiv_rn(x, a.temperature);
    }
    v[r] = x;
    mx = fmaxf(mx, x);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if (lane == 0) sm.red_f[warp] = mx;
  __syncthreads();
  if (t < CL) {
    float m = sm.red_f[0];
    for (int w = 1; w < kWarps; ++w) m = fmaxf(m, sm.red_f[w]);
    st_dsmem_f32(mapa_shared(smem_addr(&sm.cl_max[rank]), t), m);
  }
  cluster_sync_all();
  mx = sm.cl_max[0];
#pragma unroll
  for (int c = 1; c < CL; ++c) mx = fmaxf(mx, sm.cl_max[c]);
  float* E = cl_exp_buf<kSliceElems>(sm);
#pragma unroll
  for (int r = 0; r < PT; ++r) {
    const int j = t + r * kSamplerThreads;
    if (j < nloc) E[j] = __double2float_rn(exp(static_cast<double>(__fsub_rn(v[r], mx))));
  }
  cluster_sync_all();  // every slice's exponentials are readable
  stamp(1);

  // ---- normalise: p /= p.sum() (ref :51), the pairwise leaves spread ----
  tree_split(sm, V);
  const uint32_t e_base = smem_addr(E);
  tree_leaves(
      sm,
      [&](int i) {
        return ld_dsmem_f32(mapa_shared(e_base + 4u * static_cast<uint32_t>(i % kSliceElems), i / kSliceElems));
      },
      [&](int s0) { return s0 >= i0 && s0 < i0 + nloc; },
      [&](int nd, float v) {
#pragma unroll
        for (int c = 0; c < CL; ++c) st_dsmem_f32(mapa_shared(smem_addr(&sm.node_val[nd]), c), v);
      });
  cluster_sync_all();
  const float S = tree_combine(sm);
  uint64_t* X = cl_sort_buf<kSliceElems>(sm, 0);
  uint32_t kand = 0xffffffffu, kor = 0u;
#pragma unroll
  for (int r = 0; r < PT; ++r) {
    const int j = t + r * kSamplerThreads;
    if (j < nloc) {
      const uint32_t key = ~__float_as_uint(__fdiv_rn(E[j], S));  // ascending keys = descending p
      X[j] = (static_cast<uint64_t>(key) << 32) | static_cast<uint32_t>(i0 + j);
      kand &= key;
      kor |= key;
    }
  }
  kand = __reduce_and_sync(0xffffffffu, kand);
  kor = __reduce_or_sync(0xffffffffu, kor);
  if (lane == 0) {
    sm.red_and[warp] = kand;
    sm.red_or[warp] = kor;
  }
  __syncthreads();  // X and the AND / OR partials are complete
  stamp(2);

  // ---- top-p (ref :53-63): stable radix sort by (descending p, ascending id) ----
  const uint32_t below = (1u << lane) - 1u;
  int cur = 0;
  uint32_t skip = 0;  // passes whose digit every key shares (known after pass 0's exchange)
  for (int pass = 0; pass < 8; ++pass) {
    if ((skip >> pass) & 1u) continue;
    const int sh = 4 * pass;
    const uint64_t* src = cl_sort_buf<kSliceElems>(sm, cur);
    const uint32_t dst_base = smem_addr(cl_sort_buf<kSliceElems>(sm, cur ^ 1));
    uint64_t* stage = cl_sort_buf<kSliceElems>(sm, 2);  // the exponentials' space, free from here
    // this warp's positions: 4 rounds of 32 consecutive ones, in order
    uint64_t e[PT];
    if (lane < 16) sm.rs_cnt[warp][lane] = 0;
    __syncwarp();
#pragma unroll
    for (int r = 0; r < PT; ++r) {
      const int j = WPOS * warp + 32 * r + lane;
      e[r] = j < nloc ? src[j] : 0ull;
      if (j < nloc) atomicAdd(&sm.rs_cnt[warp][static_cast<uint32_t>(e[r] >> (32 + sh)) & 15u], 1);
    }
    __syncthreads();
    if (warp < 16) {  // digit d = warp: exclusive scan of the warps' counts (lane = warp index)
      const int c = sm.rs_cnt[lane][warp];
      int incl = c;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      sm.rs_off[lane][warp] = incl - c;
      if (lane == 31) sm.cl_tot[warp] = incl;
    }
    __syncthreads();
    if (warp == 0) {  // in the stage, digit d's elements of warp w start at cl_lstart[d] + rs_off[w][d]
      const int tot = lane < 16 ? sm.cl_tot[lane] : 0;
      int incl = tot;
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane < 16) {
        sm.cl_lstart[lane] = incl - tot;
#pragma unroll
        for (int c = 0; c < CL; ++c)
          st_dsmem_u32(mapa_shared(smem_addr(&sm.cl_cnt[rank][lane]), c), static_cast<uint32_t>(tot));
      }
      if (pass == 0 && lane >= 16 && lane < 16 + CL) {
        uint32_t ka = 0xffffffffu, ko = 0u;
        for (int w = 0; w < kWarps; ++w) {
          ka &= sm.red_and[w];
          ko |= sm.red_or[w];
        }
        st_dsmem_u32(mapa_shared(smem_addr(&sm.cl_and[rank]), lane - 16), ka);
        st_dsmem_u32(mapa_shared(smem_addr(&sm.cl_or[rank]), lane - 16), ko);
      }
    }
    __syncthreads();
    // stable counting sort of this CTA's elements by digit into the stage, so
    // that each digit's elements leave as one run of consecutive positions
#pragma unroll
    for (int r = 0; r < PT; ++r) {
      const int j = WPOS * warp + 32 * r + lane;
      const bool ok = j < nloc;
      const uint32_t d = static_cast<uint32_t>(e[r] >> (32 + sh)) & 15u;
      const uint32_t m = same_digit_lanes(d) & __ballot_sync(0xffffffffu, ok);
      const int pos = ok ? sm.cl_lstart[d] + sm.rs_off[warp][d] + __popc(m & below) : 0;
      __syncwarp();
      if (ok && (m & below) == 0) sm.rs_off[warp][d] += __popc(m);  // the group's lowest lane advances it
      __syncwarp();
      if (ok) stage[pos] = e[r];
    }
    cluster_sync_all();  // every CTA's digit totals (and, at pass 0, AND / OR) have arrived; the stage is complete
    if (pass == 0) {
      uint32_t ka = 0xffffffffu, ko = 0u;
#pragma unroll
      for (int c = 0; c < CL; ++c) {
        ka &= sm.cl_and[c];
        ko |= sm.cl_or[c];
      }
      const uint32_t diff = ka ^ ko;  // bits that differ between some keys
#pragma unroll
      for (int q = 1; q < 8; ++q)
        if (((diff >> (4 * q)) & 15u) == 0u) skip |= 1u << q;
    }
    if (warp == 0) {  // global start of digit d from this CTA: all smaller digits, then earlier CTAs
      int before = 0, total = 0;
      if (lane < 16)
        for (int c = 0; c < CL; ++c) {
          const int n = sm.cl_cnt[c][lane];
          if (c < rank) before += n;
          total += n;
        }
      int incl = total;
#pragma unroll
      for (int o = 1; o < 16; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      if (lane < 16) sm.cl_gofs[lane] = incl - total + before - sm.cl_lstart[lane];
    }
    __syncthreads();
#pragma unroll
    for (int r = 0; r < PT; ++r) {  // consecutive stage positions -> consecutive global positions
      const int j = t + r * kSamplerThreads;
      if (j < nloc) {
        const uint64_t x = stage[j];
        const int dst = sm.cl_gofs[static_cast<uint32_t>(x >> (32 + sh)) & 15u] + j;
        st_dsmem_u64(mapa_shared(dst_base + 8u * static_cast<uint32_t>(dst % kSliceElems), dst / kSliceElems), x);
      }
    }
    cluster_sync_all();  // the pass's output is complete in every CTA
    cur ^= 1;
  }

  // ---- gather the sorted slices into CTA 0 ----
  const uint64_t* fin = cl_sort_buf<kSliceElems>(sm, cur);
  uint64_t g[PT];
#pragma unroll
  for (int r = 0; r < PT; ++r) {
    const int j = t + r * kSamplerThreads;
    g[r] = j < nloc ? fin[j] : 0ull;
  }
  cluster_sync_all();  // CTA 0's sort buffers are free from here
  const uint32_t kb = smem_addr(sm.key), ib = smem_addr(sm.idx);
#pragma unroll
  for (int r = 0; r < PT; ++r) {
    const int j = t + r * kSamplerThreads;
    if (j < nloc) {
      const uint32_t i = static_cast<uint32_t>(i0 + j);
      st_dsmem_u32(mapa_shared(kb + 4u * i, 0), static_cast<uint32_t>(g[r] >> 32));
      st_dsmem_u16(mapa_shared(ib + 2u * i, 0), static_cast<uint32_t>(g[r]) & 0xffffu);
    }
  }
  if (lead)
    for (int i = V + t; i < kSamplerMaxVocab; i += kSamplerThreads) {
      sm.key[i] = 0xffffffffu;  // decodes to p = 0
      sm.idx[i] = 0xffff;
    }
  cluster_sync_all();  // CTA 0 holds every sorted key; the others are done
  if (!lead) return;
  stamp(3);
  int n_rounds = 0;
  const int cut = topp_cutoff(sm, V, a.top_p, a.trace != nullptr ? a.trace + static_cast<size_t>(b) * 8 + 7 : nullptr, n_rounds);
  if (a.trace != nullptr && t == 0)
    a.trace[static_cast<size_t>(b) * 8 + 6] = static_cast<uint64_t>(cut) | (static_cast<uint64_t>(n_rounds) << 32);
  stamp(4);
  const float S2 = pairwise_sum(sm, cut, [&](int i) { return key_to_p(sm.key[i]); });
  for (int i = t; i < cut; i += kSamplerThreads)  // the renormalised kept p, once each
    sm.key[i] = __float_as_uint(__fdiv_rn(key_to_p(sm.key[i]), S2));
  __syncthreads();
  const int k = cdf_search(sm, cut, a.uniforms[b], [&](int i) { return __uint_as_float(sm.key[i]); });
  if (t == 0) a.out[b] = sm.idx[k];
  stamp(5);
}

// Clusters of CL CTAs of the cluster sampler that fit co-resident on the
// current device (0 if none, or if the device refuses the cluster size);
// cached per device.  Clusters of 16 are a non-portable size: the device
// decides whether it runs them.
template <int CL>
inline int sampler_cluster_capacity() {
  static int cap[64];
  static bool known[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  if (known[dev]) return cap[dev];
  int n = 0;
  bool ok = cudaFuncSetAttribute(sample_cluster_kernel<CL>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 static_cast<int>(sizeof(SamplerSmem))) == cudaSuccess;
  if (ok && CL > 8)
    ok = cudaFuncSetAttribute(sample_cluster_kernel<CL>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) ==
         cudaSuccess;
  if (ok) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = CL;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 1;
    cfg.gridDim = dim3(CL * 32);
    cfg.blockDim = dim3(kSamplerThreads);
    cfg.dynamicSmemBytes = sizeof(SamplerSmem);
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (cudaOccupancyMaxActiveClusters(&n, sample_cluster_kernel<CL>, &cfg) != cudaSuccess) n = 0;
  }
  cudaGetLastError();
  cap[dev] = n;
  known[dev] = true;
  return n;
}

template <int CL>
inline cudaError_t launch_sampler_cluster(const SampleArgs& a, int batch, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(batch * CL));
  cfg.blockDim = dim3(kSamplerThreads);
  cfg.dynamicSmemBytes = sizeof(SamplerSmem);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = CL;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, sample_cluster_kernel<CL>, a);
}

// Kernel choice for top-p draws (mode): 0 automatic, clusters of 16 CTAs per
// sequence where every cluster of the batch is co-resident, else of 8, else one
// CTA per sequence; 1 one CTA per sequence; 2 clusters of 8 where they fit.
inline cudaError_t launch_sampler(const float* logits, int batch, int vocab, const int32_t* history,
                                  int hist_cap, const int32_t* hist_len, const double* uniforms,
                                  double temperature, double top_p, double rep_penalty, int32_t* out,
                                  cudaStream_t st, uint64_t* scratch, uint64_t* trace = nullptr,
                                  int mode = 0) {
  static bool attr_set[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!attr_set[dev]) {
    e = cudaFuncSetAttribute(sample_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(sizeof(SamplerSmem)));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  SampleArgs a;
  a.logits = logits;
  a.history = history;
  a.hist_len = hist_len;
  a.uniforms = uniforms;
  a.out = out;
  a.vocab = vocab;
  a.hist_cap = hist_cap;
  a.temperature = static_cast<float>(temperature);
  a.rep_penalty = static_cast<float>(rep_penalty);
  a.top_p = top_p;
  a.trace = trace;
  a.scratch = scratch;
  // top-p draws go to a cluster kernel when every sequence's cluster is
  // co-resident (one wave); larger batches keep one CTA per sequence
  if (mode != 1 && a.temperature > 0.0f && top_p < 1.0) {
    if (mode == 0 && batch <= sampler_cluster_capacity<16>()) return launch_sampler_cluster<16>(a, batch, st);
    if (batch <= sampler_cluster_capacity<8>()) return launch_sampler_cluster<8>(a, batch, st);
  }
  sample_kernel<<<batch, kSamplerThreads, sizeof(SamplerSmem), st>>>(a);
  return cudaGetLastError();
}

}  // namespace b2d
