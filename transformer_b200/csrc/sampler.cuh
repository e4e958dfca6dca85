// sampler.cuh — device sampler, one CTA per sequence (sm_100a).
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
//   * top-p: order by descending probability, ties by ascending token id; the
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

namespace b2d {

constexpr int kSamplerMaxVocab = 32768;
constexpr int kSamplerThreads = 1024;
constexpr int kTreeNodes = 1024;  // heap-indexed pairwise-sum tree (depth <= 9)

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
};

__device__ __forceinline__ float key_to_p(uint32_t k) { return __uint_as_float(~k); }

// numpy's pairwise float32 sum of get(0..n-1), evaluated level by level over
// a heap-indexed tree of its recursion; returns 0 + sum like np.sum.  All
// threads of the block must call it.
template <class Get>
__device__ float pairwise_sum(SamplerSmem& sm, int n, Get get) {
  const int t = threadIdx.x;
  if (t == 0) {
    for (int i = 0; i < kTreeNodes; ++i) sm.node_len[i] = -1;
    sm.node_start[1] = 0;
    sm.node_len[1] = n;
  }
  __syncthreads();
  // top-down: split every node longer than 128 (n2 = n/2 rounded down to 8)
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
  // leaves (len <= 128): numpy's 8-accumulator block sum
  for (int nd = 1 + t; nd < kTreeNodes; nd += blockDim.x) {
    const int len = sm.node_len[nd];
    if (len < 0 || len > 128) continue;
    const int s0 = sm.node_start[nd];
    float res;
    if (len < 8) {
      res = 0.f;
      for (int i = 0; i < len; ++i) res = __fadd_rn(res, get(s0 + i));
    } else {
      float r[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) r[j] = get(s0 + j);
      int i = 8;
      for (; i < len - (len % 8); i += 8) {
#pragma unroll
        for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], get(s0 + i + j));
      }
      res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                      __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
      for (; i < len; ++i) res = __fadd_rn(res, get(s0 + i));
    }
    sm.node_val[nd] = res;
  }
  __syncthreads();
  // bottom-up: internal node = left + right
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

// Block-wide float64 prefix sums of get(0..n-1) (thread-contiguous chunks);
// returns the first k with prefix_k / total > u (numpy's searchsorted 'right'
// after cdf /= cdf[-1]).
template <class Get>
__device__ int cdf_search(SamplerSmem& sm, int n, double u, Get get) {
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int per = (n + kSamplerThreads - 1) / kSamplerThreads;
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
  double run = (warp > 0 ? sm.red_d[warp - 1] : 0.0) + (incl - local);
  int found = 0x7fffffff;
  for (int i = i0; i < i1; ++i) {
    run += static_cast<double>(get(i));
    if (run / total > u) { found = i; break; }
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

// Bitonic compare-exchange of (k, x) pairs: ascending by (key, id) when asc.
__device__ __forceinline__ void cmp_swap(uint32_t& ka, uint32_t& xa, uint32_t& kb, uint32_t& xb, bool asc) {
  const bool sw = (ka > kb || (ka == kb && xa > xb)) == asc;  // (branch-free)
  const uint32_t k0 = sw ? kb : ka, k1 = sw ? ka : kb, x0 = sw ? xb : xa, x1 = sw ? xa : xb;
  ka = k0; kb = k1; xa = x0; xb = x1;
}

// Bitonic steps with partner distance j < kSortChunk for stages kk_lo ..
// kk_hi (powers of two) on every chunk of kSortChunk consecutive elements,
// in registers; element e of a stage kk sorts ascending iff (e & kk) == 0.
// A thread reads its chunk's 16-byte pieces starting at a rotation of its
// own (conflict-free across the warp) and undoes the rotation with selects.
constexpr int kSortChunk = 16;
__device__ __forceinline__ void sort_chunks(SamplerSmem& sm, int kk_lo, int kk_hi) {
  const int rk = (threadIdx.x >> 1) & 3, rx = (threadIdx.x >> 2) & 1;  // rotations of the key / id pieces
  for (int c = threadIdx.x; c < kSamplerMaxVocab / kSortChunk; c += kSamplerThreads) {
    const int base = c * kSortChunk;
    uint32_t k[kSortChunk], x[kSortChunk];
    {
      const uint4* k4 = reinterpret_cast<const uint4*>(sm.key + base);
      uint4 v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = k4[(q + rk) & 3];  // v[q] = piece (q + rk) & 3
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // piece q = v[(q - rk) & 3]
        const uint4 a0 = v[q], a1 = v[(q + 3) & 3], a2 = v[(q + 2) & 3], a3 = v[(q + 1) & 3];
        const uint4 w = rk == 0 ? a0 : rk == 1 ? a1 : rk == 2 ? a2 : a3;
        k[4 * q] = w.x; k[4 * q + 1] = w.y; k[4 * q + 2] = w.z; k[4 * q + 3] = w.w;
      }
      const uint4* x4 = reinterpret_cast<const uint4*>(sm.idx + base);  // 8 ids per piece
      const uint4 y0 = x4[rx], y1 = x4[rx ^ 1];
      const uint4 p0 = rx ? y1 : y0, p1 = rx ? y0 : y1;
      const uint32_t wv[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
      for (int h = 0; h < 8; ++h) {
        x[2 * h] = wv[h] & 0xffffu;
        x[2 * h + 1] = wv[h] >> 16;
      }
    }
    for (int kk = kk_lo; kk <= kk_hi; kk <<= 1) {
#pragma unroll
      for (int j = kSortChunk / 2; j > 0; j >>= 1) {
        if (j >= kk) continue;  // stage kk has steps j = kk/2 .. 1
#pragma unroll
        for (int e = 0; e < kSortChunk; ++e)
          if (!(e & j)) cmp_swap(k[e], x[e], k[e + j], x[e + j], ((base + e) & kk) == 0);
      }
    }
    {
      uint4 v[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) v[q] = make_uint4(k[4 * q], k[4 * q + 1], k[4 * q + 2], k[4 * q + 3]);
      uint4* k4 = reinterpret_cast<uint4*>(sm.key + base);
#pragma unroll
      for (int q = 0; q < 4; ++q) {  // store piece (q + rk) & 3
        const uint4 a0 = v[q], a1 = v[(q + 1) & 3], a2 = v[(q + 2) & 3], a3 = v[(q + 3) & 3];
        k4[(q + rk) & 3] = rk == 0 ? a0 : rk == 1 ? a1 : rk == 2 ? a2 : a3;
      }
      const uint4 p0 = make_uint4(x[0] | (x[1] << 16), x[2] | (x[3] << 16), x[4] | (x[5] << 16), x[6] | (x[7] << 16));
      const uint4 p1 = make_uint4(x[8] | (x[9] << 16), x[10] | (x[11] << 16), x[12] | (x[13] << 16),
                                  x[14] | (x[15] << 16));
      uint4* x4 = reinterpret_cast<uint4*>(sm.idx + base);
      x4[rx] = rx ? p1 : p0;
      x4[rx ^ 1] = rx ? p0 : p1;
    }
  }
  __syncthreads();
}

// S consecutive bitonic steps of stage kk with distances jtop, jtop/2, ..,
// d = jtop / 2^(S-1) (>= kSortChunk) in one shared-memory pass: a thread
// loads groups of 2^S elements base + a*d, applies the S steps in registers
// and stores them back.
template <int S>
__device__ __forceinline__ void sort_group_pass(SamplerSmem& sm, int kk, int jtop) {
  constexpr int G = 1 << S;
  const int d = jtop >> (S - 1), ld = __ffs(d) - 1;
#pragma unroll 1
  for (int gi = threadIdx.x; gi < kSamplerMaxVocab / G; gi += kSamplerThreads) {
    const int base = ((gi >> ld) << (ld + S)) | (gi & (d - 1));
    uint32_t k[G], x[G];
#pragma unroll
    for (int a = 0; a < G; ++a) {
      k[a] = sm.key[base + a * d];
      x[a] = sm.idx[base + a * d];
    }
    const bool asc = (base & kk) == 0;  // a*d < 2*jtop <= kk adds no carry into bit kk
#pragma unroll
    for (int m = G / 2; m > 0; m >>= 1)
#pragma unroll
      for (int a = 0; a < G; ++a)
        if (!(a & m)) cmp_swap(k[a], x[a], k[a + m], x[a + m], asc);
#pragma unroll
    for (int a = 0; a < G; ++a) {
      sm.key[base + a * d] = k[a];
      sm.idx[base + a * d] = static_cast<uint16_t>(x[a]);
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kSamplerThreads, 1) sample_kernel(const SampleArgs a) {
  extern __shared__ __align__(16) uint8_t sampler_smem_raw[];
  SamplerSmem& sm = *reinterpret_cast<SamplerSmem*>(sampler_smem_raw);
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int V = a.vocab;
  const float* lg = a.logits + static_cast<size_t>(b) * V;
  constexpr int PER = kSamplerMaxVocab / kSamplerThreads;
  // stamps: 0 entry, 1 exponentials, 2 normalised, 3 sorted, 4 cutoff, 5 drawn
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
  // Bitonic sort ascending by (key, id) (key = ~bits of p).  Steps whose
  // partner distance j < kSortChunk stay inside a thread's chunk of
  // kSortChunk consecutive elements and run in registers; wider steps are
  // shared-memory passes with every load of a batch issued before its stores.
  stamp(2);
  sort_chunks(sm, 2, kSortChunk);  // stages kk = 2 .. kSortChunk entirely in registers
  for (int kk = 2 * kSortChunk; kk <= kSamplerMaxVocab; kk <<= 1) {
    // steps j = kk/2 .. kSortChunk, up to 4 per shared-memory pass
    for (int j = kk >> 1; j >= kSortChunk;) {
      const int left = __ffs(j) - __ffs(kSortChunk) + 1;  // steps j .. kSortChunk
      if (left >= 4) { sort_group_pass<4>(sm, kk, j); j >>= 4; }
      else if (left == 3) { sort_group_pass<3>(sm, kk, j); j >>= 3; }
      else if (left == 2) { sort_group_pass<2>(sm, kk, j); j >>= 2; }
      else { sort_group_pass<1>(sm, kk, j); j >>= 1; }
    }
    sort_chunks(sm, kk, kk);  // this stage's steps j < kSortChunk, in registers
  }
  stamp(3);
  // cutoff = first k with float64(cumsum_f32[k]) >= top_p, plus one.  The
  // running sum is a float, so float64(c) >= top_p  <=>  c >= thr with thr =
  // top_p rounded up to a float: the chain stays in float32 (the cumulative
  // sum itself is sequential, as numpy's).
  if (t == 0) {  // one thread runs the float32 chain in order, 16 keys per block
    const float thr = __double2float_ru(a.top_p);
    const uint4* k4 = reinterpret_cast<const uint4*>(sm.key);
    const int n4 = (V + 3) / 4;  // keys past V decode to p = 0
    constexpr int Q = 4;         // uint4 per block
    auto load_blk = [&](int base, uint4 (&dst)[Q]) {
#pragma unroll
      for (int q = 0; q < Q; ++q) dst[q] = base + q < n4 ? k4[base + q] : make_uint4(~0u, ~0u, ~0u, ~0u);
    };
    float c = 0.f;
    int cut = V;
    uint4 nxt[Q];
    load_blk(0, nxt);
    for (int base = 0; base < n4; base += Q) {
      uint4 cur[Q];
#pragma unroll
      for (int q = 0; q < Q; ++q) cur[q] = nxt[q];
      load_blk(base + Q, nxt);  // the next block's keys are in flight during this block's chain
      // The sum never decreases (p >= 0): the threshold is crossed inside this
      // block iff it is crossed at its end; only then is the block rerun key by key.
      float e = c;
#pragma unroll
      for (int q = 0; q < Q; ++q) {
        e = __fadd_rn(e, key_to_p(cur[q].x));
        e = __fadd_rn(e, key_to_p(cur[q].y));
        e = __fadd_rn(e, key_to_p(cur[q].z));
        e = __fadd_rn(e, key_to_p(cur[q].w));
      }
      if (e >= thr) {
        for (int i = 0; i < 4 * Q; ++i) {
          c = __fadd_rn(c, 4 * base + i < V ? key_to_p(sm.key[4 * base + i]) : 0.f);
          if (c >= thr) {
            cut = 4 * base + i + 1;
            break;
          }
        }
        break;
      }
      c = e;
    }
    sm.cutoff = min(cut, V);
  }
  __syncthreads();
  const int cut = sm.cutoff;
  stamp(4);
  const float S2 = pairwise_sum(sm, cut, [&](int i) { return key_to_p(sm.key[i]); });
  const int k = cdf_search(sm, cut, a.uniforms[b], [&](int i) { return __fdiv_rn(key_to_p(sm.key[i]), S2); });
  if (t == 0) a.out[b] = sm.idx[k];
  stamp(5);
}

inline cudaError_t launch_sampler(const float* logits, int batch, int vocab, const int32_t* history,
                                  int hist_cap, const int32_t* hist_len, const double* uniforms,
                                  double temperature, double top_p, double rep_penalty, int32_t* out,
                                  cudaStream_t st, uint64_t* trace = nullptr) {
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
  sample_kernel<<<batch, kSamplerThreads, sizeof(SamplerSmem), st>>>(a);
  return cudaGetLastError();
}

}  // namespace b2d
