// batched.cuh — the batched decode step's non-GEMM kernels (sm_100a).
//
// The batched step runs, per layer: RMSNorm -> QKV
// projection -> paged attention (RoPE, K/V append, GQA attention) -> O
// projection + residual -> RMSNorm -> gate/up projection + SwiGLU -> down
// projection + residual; the projections are the tensor-core kernel of
// gemm_tc.cuh, these kernels are the rest.  Math follows the reference
// (model.py:94-191; RMSNorm output and attention output rounded to bf16 before
// their projections as in kernels/multi_sm_decode.py:133-152 and :229).
//
// A sequence with pos < 0 is inactive for the step: nothing is written to its
// cache and its outputs are meaningless (used to ingest ragged prompts).
//
// Paged KV pool layout (bf16): [layer][block][K|V][kv_head][16][64], K
// post-RoPE; block_table[b][i] is the physical block of positions
// 16i..16i+15 of sequence b.
#pragma once

#include <cuda_bf16.h>

#include "b2d_ptx.cuh"

namespace b2d {

constexpr int kPageTokens = 16;

// H[b][:] = f32(emb[tok[b]]);  X[b][:] = bf16(RMSNorm(H[b]) * g)  (model.py:94-98,
// layer 0's ln1).  One CTA (256 threads) per row; fixed-order reduction.
__global__ void embed_rows_kernel(const __nv_bfloat16* __restrict__ emb, const int32_t* __restrict__ tok,
                                  int vocab, int D, const float* __restrict__ g, float eps, float* __restrict__ H,
                                  __nv_bfloat16* __restrict__ X, uint32_t* status) {
  __shared__ float red[8];
  pdl_wait();
  pdl_launch();
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  int tk = tok[b];
  if (tk < 0 || tk >= vocab) {
    if (t == 0) atomicCAS(status, 0u, 0x201u);
    tk = 0;
  }
  const __nv_bfloat16* e = emb + static_cast<size_t>(tk) * D;
  float* h = H + static_cast<size_t>(b) * D;
  float ss = 0.f;
  for (int i = t; i < D; i += 256) {
    const float v = __bfloat162float(e[i]);
    h[i] = v;
    ss = fmaf(v, v, ss);
  }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float r = rsqrtf(tot / static_cast<float>(D) + eps);
  for (int i = t; i < D; i += 256)
    X[static_cast<size_t>(b) * D + i] = __float2bfloat16_rn(__bfloat162float(e[i]) * r * __ldg(g + i));
}

// X[b][:] = bf16(H[b] * rsqrt(mean(H[b]^2) + eps) * g)   (model.py:94-98)
// One CTA (128 threads) per row, the row held in registers (D <= 2048,
// D % 4 == 0); fixed-order reduction.
__global__ void __launch_bounds__(128) rmsnorm_rows_kernel(const float* __restrict__ H, const float* __restrict__ g,
                                                           int D, float eps, __nv_bfloat16* __restrict__ X) {
  __shared__ float red[4];
  pdl_wait();
  pdl_launch();
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float4* h = reinterpret_cast<const float4*>(H + static_cast<size_t>(b) * D);
  const int q4 = D / 4;  // float4s per row, <= 4 per thread
  float4 v[4] = {};
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (t + 128 * i < q4) {
      v[i] = h[t + 128 * i];
      ss = fmaf(v[i].x, v[i].x, ss); ss = fmaf(v[i].y, v[i].y, ss);
      ss = fmaf(v[i].z, v[i].z, ss); ss = fmaf(v[i].w, v[i].w, ss);
    }
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  const float r = rsqrtf((red[0] + red[1] + red[2] + red[3]) / static_cast<float>(D) + eps);
  const float4* g4 = reinterpret_cast<const float4*>(g);
  __nv_bfloat162* x = reinterpret_cast<__nv_bfloat162*>(X + static_cast<size_t>(b) * D);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (t + 128 * i < q4) {
      const float4 w = __ldg(g4 + t + 128 * i);
      x[2 * (t + 128 * i)] = __floats2bfloat162_rn(v[i].x * r * w.x, v[i].y * r * w.y);
      x[2 * (t + 128 * i) + 1] = __floats2bfloat162_rn(v[i].z * r * w.z, v[i].w * r * w.w);
    }
}

struct PagedAttnArgs {
  const float* qkv;            // [B][(H+2KVH)*64] f32 (pre-RoPE q, k; v)
  const int32_t* pos;          // [B]
  __nv_bfloat16* pool;         // paged KV pool
  const int32_t* table;        // [B][bps]
  int bps, num_blocks, layer, n_heads, n_kv, ctx;
  const float* rcos;           // [ctx][32]
  const float* rsin;
  __nv_bfloat16* out;          // [B][ldo] bf16: head h at columns h*64..
  int ldo;
  uint32_t* status;            // set when a block-table entry is out of range
  float* part;                 // [B][n_heads][max_chunks][kAttPart] per-CTA partials
  uint32_t* tickets;           // [B][n_kv]; zero between launches (the combining CTA resets it)
  int max_chunks;              // >= ceil(ctx / kAttChunk)
  int cpc;                     // chunks per CTA (>= 1)
  // Cache addressing: table != nullptr -> the paged pool above; table ==
  // nullptr -> one sequence's contiguous cache in the reference layout
  // [layer][K|V][kv_head][ctx][64] (every row of the launch is a position of
  // that sequence, as in a prefill).
  bool append;                 // the CTA holding a row's position writes its K/V (else done before)
};

// K (kv = 0) or V (kv = 1) row of position `pos` of the launch row's sequence.
__device__ __forceinline__ __nv_bfloat16* kv_row(const PagedAttnArgs& a, const int32_t* tb, int pos, int kv, int g) {
  if (a.table == nullptr)
    return a.pool + ((((static_cast<size_t>(a.layer) * 2 + kv) * a.n_kv + g) * a.ctx) + pos) * 64;
  return a.pool + ((((static_cast<size_t>(a.layer) * a.num_blocks + tb[pos / kPageTokens]) * 2 + kv) * a.n_kv + g) *
                       kPageTokens + pos % kPageTokens) * 64;
}

// Writes row b's K (post-RoPE) / V for kv head blockIdx.y at position pos[b]
// (bf16, as cached).  grid (rows, n_kv), 32 threads.  Used before a prefill
// launch of the attention (append = false) so that every row's K/V is in the
// cache before any row attends.  Positions out of range / idle rows: skipped.
__global__ void __launch_bounds__(32) kv_append_kernel(const __grid_constant__ PagedAttnArgs a) {
  pdl_wait();
  pdl_launch();
  const int b = blockIdx.x, g = blockIdx.y, lane = threadIdx.x;
  const int p = a.pos[b];
  if (p < 0 || p >= a.ctx) return;
  const int32_t* tb = a.table ? a.table + static_cast<size_t>(b) * a.bps : nullptr;
  if (tb != nullptr) {
    if (p / kPageTokens >= a.bps) return;
    const int e = tb[p / kPageTokens];
    if (e < 0 || e >= a.num_blocks) {
      if (lane == 0) atomicCAS(a.status, 0u, 0x203u);
      return;
    }
  }
  const float* row = a.qkv + static_cast<size_t>(b) * (a.n_heads + 2 * a.n_kv) * 64;
  const float cs = a.rcos[static_cast<size_t>(p) * 32 + lane], sn = a.rsin[static_cast<size_t>(p) * 32 + lane];
  const float* k = row + a.n_heads * 64 + g * 64;
  const float* v = row + (a.n_heads + a.n_kv) * 64 + g * 64;
  const float klo = k[lane], khi = k[lane + 32];
  __nv_bfloat16* kd = kv_row(a, tb, p, 0, g);
  __nv_bfloat16* vd = kv_row(a, tb, p, 1, g);
  kd[lane] = __float2bfloat16_rn(klo * cs - khi * sn);
  kd[lane + 32] = __float2bfloat16_rn(klo * sn + khi * cs);
  vd[lane] = __float2bfloat16_rn(v[lane]);
  vd[lane + 32] = __float2bfloat16_rn(v[lane + 32]);
}

constexpr int kAttChunk = 64;  // cached positions per CTA
constexpr int kAttPart = 68;   // m, l, 2 pad, o[64]
constexpr int kAttRow = 72;    // smem row pitch (bf16): 144 B keeps 16-byte row reads conflict-free


// Split ("flash-decoding") paged attention.  grid (ceil(max_chunks / cpc),
// n_kv, B), block 128: CTA (x, g, b) handles the cached positions of chunks
// x*cpc .. x*cpc+cpc-1 (64 positions each) of sequence b for the GQA query
// heads of kv head g (GQA <= 4), merging its chunks with an online softmax;
// the next chunk's K/V loads are in flight while the current chunk is
// computed.  The CTA holding the new position appends its K (post-RoPE) / V
// to the pool.  K/V rows are staged in padded shared memory and every
// element is read and converted once for all the GQA heads: scores by
// (position, half of the dimensions), P.V by (dimension pair, group of 16
// positions), packed f32x2 FMAs.  When a sequence spans several CTAs each
// writes (m, l, o) and the last to finish (ticket) merges them in CTA order
// and writes the bf16 output.  Math: model.py:100-131 (rotate-half RoPE,
// causal softmax over 0..p, GQA sharing).
__global__ void __launch_bounds__(128) paged_attn_kernel(const __grid_constant__ PagedAttnArgs a) {
  __shared__ __align__(16) __nv_bfloat16 sk[kAttChunk][kAttRow];
  __shared__ __align__(16) __nv_bfloat16 sv[kAttChunk][kAttRow];
  __shared__ __align__(16) float sq[4][2][36];      // q by head and half of the dims (padded: no bank clash)
  __shared__ __align__(16) float ss[kAttChunk][4];  // probabilities by position and head
  __shared__ float smax[4][4], ssum[4][4];          // per warp, per head
  __shared__ __align__(16) float sacc[4][4][64];    // P.V partials by position group, head, dim
  __shared__ __align__(16) __nv_bfloat16 skn[64], svn[64];  // the new position's K / V
  __shared__ uint32_t s_last;
  const int x = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int GQA = a.n_heads / a.n_kv;
  pdl_wait();
  pdl_launch();
  const int p = a.pos[b];
  if (p < 0 || p >= a.ctx) {  // idle sequence: no cache write, zero output
    if (x == 0 && warp < GQA)
      reinterpret_cast<__nv_bfloat162*>(a.out + static_cast<size_t>(b) * a.ldo + (g * GQA + warp) * 64)[lane] =
          __floats2bfloat162_rn(0.f, 0.f);
    return;
  }
  const int nch = p / kAttChunk + 1;
  const int c_lo = x * a.cpc;
  if (c_lo >= nch) return;
  const int c_hi = min(c_lo + a.cpc, nch);
  const int ncta = (nch + a.cpc - 1) / a.cpc;  // CTAs sharing this (b, g)
  const int32_t* tb = a.table ? a.table + static_cast<size_t>(b) * a.bps : nullptr;
  // every page this CTA touches must exist (paged cache)
  bool bad = tb != nullptr && (p / kPageTokens) >= a.bps;
  const int pg_hi = (min(c_hi * kAttChunk, p + 1) - 1) / kPageTokens;
  for (int i = c_lo * (kAttChunk / kPageTokens) + t; tb != nullptr && !bad && i <= pg_hi; i += 128) {
    const int e = tb[i];
    bad = e < 0 || e >= a.num_blocks;
  }
  bad = __syncthreads_or(bad);
  if (bad && t == 0) atomicCAS(a.status, 0u, 0x203u);

  const float* row = a.qkv + static_cast<size_t>(b) * (a.n_heads + 2 * a.n_kv) * 64;
  const bool owner = c_hi == nch;  // this CTA's last chunk holds position p
  if (t < 32) {
    const float cs = a.rcos[static_cast<size_t>(p) * 32 + lane], sn = a.rsin[static_cast<size_t>(p) * 32 + lane];
#pragma unroll
    for (int w = 0; w < 4; ++w) {  // RoPE (rotate-half); q pre-scaled by 1/sqrt(64) (exact); unused heads 0
      float lo = 0.f, hi = 0.f;
      if (w < GQA) {
        const float* q = row + (g * GQA + w) * 64;
        lo = q[lane];
        hi = q[lane + 32];
      }
      sq[w][0][lane] = (lo * cs - hi * sn) * 0.125f;
      sq[w][1][lane] = (lo * sn + hi * cs) * 0.125f;
    }
    if (owner) {  // the new position's K (post-RoPE) / V, bf16 as cached
      const float* k = row + a.n_heads * 64 + g * 64;
      const float* v = row + (a.n_heads + a.n_kv) * 64 + g * 64;
      const float klo = k[lane], khi = k[lane + 32];
      skn[lane] = __float2bfloat16_rn(klo * cs - khi * sn);
      skn[lane + 32] = __float2bfloat16_rn(klo * sn + khi * cs);
      svn[lane] = __float2bfloat16_rn(v[lane]);
      svn[lane + 32] = __float2bfloat16_rn(v[lane + 32]);
      if (!bad && a.append) {
        __nv_bfloat16* kd = kv_row(a, tb, p, 0, g);
        __nv_bfloat16* vd = kv_row(a, tb, p, 1, g);
        kd[lane] = skn[lane];
        kd[lane + 32] = skn[lane + 32];
        vd[lane] = svn[lane];
        vd[lane + 32] = svn[lane + 32];
      }
    }
  }

  // thread t stages rows (t + 128 i) >> 3, 16-byte column (t + 128 i) & 7, i < 4
  uint4 kr[4] = {}, vr[4] = {};
  auto fetch = [&](int c) {
    const int base = c * kAttChunk;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = t + 128 * i, r = idx >> 3, cc = idx & 7, pp = base + r;
      if (!bad && pp < p) {
        kr[i] = __ldg(reinterpret_cast<const uint4*>(kv_row(a, tb, pp, 0, g)) + cc);
        vr[i] = __ldg(reinterpret_cast<const uint4*>(kv_row(a, tb, pp, 1, g)) + cc);
      }
    }
  };
  fetch(c_lo);
  // online-softmax state per head, the same in every thread
  float m[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY}, l[4] = {0.f, 0.f, 0.f, 0.f};
  uint64_t acc[4] = {0, 0, 0, 0};          // f32x2: dims 2*lane, 2*lane+1 of each head, this warp's 16 rows
  const int rs = t >> 1, half = t & 1;     // score mapping: row rs, dims 32*half .. 32*half+31
  for (int c = c_lo; c < c_hi; ++c) {
    const int base = c * kAttChunk;
    const int npos = min(kAttChunk, p + 1 - base);  // rows 0..npos-1 = positions base..
    __syncthreads();  // the previous chunk's reads of sk / sv / ss are done
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int idx = t + 128 * i, r = idx >> 3, cc = idx & 7, pp = base + r;
      if (pp < p) {
        *reinterpret_cast<uint4*>(&sk[r][cc * 8]) = kr[i];
        *reinterpret_cast<uint4*>(&sv[r][cc * 8]) = vr[i];
      } else if (pp == p) {
        *reinterpret_cast<uint4*>(&sk[r][cc * 8]) = reinterpret_cast<const uint4*>(skn)[cc];
        *reinterpret_cast<uint4*>(&sv[r][cc * 8]) = reinterpret_cast<const uint4*>(svn)[cc];
      } else {  // past p: zero V so the P.V rows below read finite values
        *reinterpret_cast<uint4*>(&sv[r][cc * 8]) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    __syncthreads();
    if (c + 1 < c_hi) fetch(c + 1);  // in flight during this chunk's math

    // scores: row rs, half the dimensions, all four heads; the halves meet by shuffle
    const bool valid = !bad && rs < npos;
    float sc[4] = {0.f, 0.f, 0.f, 0.f};
    if (valid) {
      uint64_t a2[4] = {0, 0, 0, 0};
      const uint4* kr4 = reinterpret_cast<const uint4*>(&sk[rs][32 * half]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint4 kw = kr4[i];
        const uint64_t k0 = bf2pack(kw.x), k1 = bf2pack(kw.y), k2 = bf2pack(kw.z), k3 = bf2pack(kw.w);
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          const float4 qa = *reinterpret_cast<const float4*>(&sq[h][half][8 * i]);
          const float4 qb = *reinterpret_cast<const float4*>(&sq[h][half][8 * i + 4]);
          a2[h] = ffma2(k0, f2pack(qa.x, qa.y), a2[h]);
          a2[h] = ffma2(k1, f2pack(qa.z, qa.w), a2[h]);
          a2[h] = ffma2(k2, f2pack(qb.x, qb.y), a2[h]);
          a2[h] = ffma2(k3, f2pack(qb.z, qb.w), a2[h]);
        }
      }
#pragma unroll
      for (int h = 0; h < 4; ++h) sc[h] = f2sum(a2[h]);
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      sc[h] += __shfl_xor_sync(0xffffffffu, sc[h], 1);
      if (!valid) sc[h] = -INFINITY;
      float mx = sc[h];
#pragma unroll
      for (int off = 16; off > 1; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (lane == 0) smax[warp][h] = mx;
    }
    __syncthreads();
    float alpha[4], pr[4];
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float mc = fmaxf(fmaxf(smax[0][h], smax[1][h]), fmaxf(smax[2][h], smax[3][h]));
      const float mn = fmaxf(m[h], mc);
      alpha[h] = m[h] == -INFINITY ? 0.f : __expf(m[h] - mn);
      pr[h] = valid ? __expf(sc[h] - mn) : 0.f;
      m[h] = mn;
      float sm = half == 0 ? pr[h] : 0.f;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, off);
      if (lane == 0) ssum[warp][h] = sm;
    }
    if (half == 0) *reinterpret_cast<float4*>(ss[rs]) = make_float4(pr[0], pr[1], pr[2], pr[3]);
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      l[h] = fmaf(l[h], alpha[h], (ssum[0][h] + ssum[1][h]) + (ssum[2][h] + ssum[3][h]));
      acc[h] = ffma2(acc[h], f2pack(alpha[h], alpha[h]), 0ull);
    }
    if (!bad) {  // P.V: dims 2*lane, 2*lane+1, rows 16*warp .. 16*warp+15, all heads
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int r = warp * 16 + i;
        const uint64_t v = bf2pack(*reinterpret_cast<const uint32_t*>(&sv[r][2 * lane]));
        const float4 p4 = *reinterpret_cast<const float4*>(ss[r]);
        acc[0] = ffma2(f2pack(p4.x, p4.x), v, acc[0]);
        acc[1] = ffma2(f2pack(p4.y, p4.y), v, acc[1]);
        acc[2] = ffma2(f2pack(p4.z, p4.z), v, acc[2]);
        acc[3] = ffma2(f2pack(p4.w, p4.w), v, acc[3]);
      }
    }
  }
  // sum the four row groups in group order; warp h < GQA then owns head g*GQA + h
#pragma unroll
  for (int h = 0; h < 4; ++h) *reinterpret_cast<uint64_t*>(&sacc[warp][h][2 * lane]) = acc[h];
  __syncthreads();
  const int h = g * GQA + warp;
  float o0 = 0.f, o1 = 0.f, mw = -INFINITY, lw = 0.f;
  if (warp < GQA) {
#pragma unroll
    for (int grp = 0; grp < 4; ++grp) {
      const float2 v = *reinterpret_cast<const float2*>(&sacc[grp][warp][2 * lane]);
      o0 += v.x;
      o1 += v.y;
    }
    mw = warp == 0 ? m[0] : warp == 1 ? m[1] : warp == 2 ? m[2] : m[3];
    lw = warp == 0 ? l[0] : warp == 1 ? l[1] : warp == 2 ? l[2] : l[3];
  }

  if (ncta == 1) {  // the whole sequence in this CTA: final output directly
    if (warp < GQA) {
      const float inv = lw > 0.f ? 1.0f / lw : 0.f;
      reinterpret_cast<__nv_bfloat162*>(a.out + static_cast<size_t>(b) * a.ldo + h * 64)[lane] =
          __floats2bfloat162_rn(o0 * inv, o1 * inv);
    }
    return;
  }
  if (warp < GQA) {
    float* part = a.part + ((static_cast<size_t>(b) * a.n_heads + h) * a.max_chunks + x) * kAttPart;
    reinterpret_cast<float2*>(part + 4)[lane] = make_float2(o0, o1);
    if (lane == 0) {
      part[0] = bad ? -INFINITY : mw;
      part[1] = lw;
    }
  }
  __threadfence();
  __syncthreads();
  if (t == 0) {
    const uint32_t prev = atomicAdd(&a.tickets[b * a.n_kv + g], 1u);
    s_last = prev == static_cast<uint32_t>(ncta - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (t == 0) a.tickets[b * a.n_kv + g] = 0u;
  if (warp < GQA) {  // merge the CTAs' partials of head h in CTA order (lane j holds CTA j's m, l)
    const float* ph = a.part + (static_cast<size_t>(b) * a.n_heads + h) * a.max_chunks * kAttPart;
    float mc = -INFINITY, lc = 0.f;
    if (lane < ncta) {
      mc = __ldcg(ph + lane * kAttPart);
      lc = __ldcg(ph + lane * kAttPart + 1);
    }
    float M = mc;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    const float wl = mc == -INFINITY ? 0.f : __expf(mc - M);
    float L = wl * lc;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    float r0 = 0.f, r1 = 0.f;
#pragma unroll 8
    for (int j = 0; j < ncta; ++j) {
      const float wgt = __shfl_sync(0xffffffffu, wl, j);
      const float2 oc = __ldcg(reinterpret_cast<const float2*>(ph + j * kAttPart + 4) + lane);
      r0 = fmaf(wgt, oc.x, r0);
      r1 = fmaf(wgt, oc.y, r1);
    }
    const float inv = L > 0.f ? 1.0f / L : 0.f;
    reinterpret_cast<__nv_bfloat162*>(a.out + static_cast<size_t>(b) * a.ldo + h * 64)[lane] =
        __floats2bfloat162_rn(r0 * inv, r1 * inv);
  }
}

// next[b] = first index of the maximum of logits[b][0..V)  (one CTA per row)
__global__ void argmax_rows_kernel(const float* __restrict__ logits, int V, int ldl, int32_t* __restrict__ next) {
  __shared__ float rv[32];
  __shared__ int ri[32];
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  pdl_wait();
  pdl_launch();
  const float* r = logits + static_cast<size_t>(b) * ldl;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int i = t; i < V; i += blockDim.x) {
    const float x = r[i];
    if (x > bv) { bv = x; bi = i; }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, off);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
  }
  if (lane == 0) { rv[warp] = bv; ri[warp] = bi; }
  __syncthreads();
  if (t == 0) {
    for (int w = 1; w < static_cast<int>(blockDim.x) / 32; ++w)
      if (rv[w] > bv || (rv[w] == bv && ri[w] < bi)) { bv = rv[w]; bi = ri[w]; }
    next[b] = bi == 0x7fffffff ? 0 : bi;
  }
}

}  // namespace b2d
