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

// H[b][:] = f32(emb[tok[b]])
__global__ void embed_rows_kernel(const __nv_bfloat16* __restrict__ emb, const int32_t* __restrict__ tok,
                                  int vocab, int D, float* __restrict__ H, uint32_t* status) {
  const int b = blockIdx.x;
  int t = tok[b];
  if (t < 0 || t >= vocab) {
    if (threadIdx.x == 0) atomicCAS(status, 0u, 0x201u);
    t = 0;
  }
  const __nv_bfloat16* e = emb + static_cast<size_t>(t) * D;
  for (int i = threadIdx.x; i < D; i += blockDim.x) H[static_cast<size_t>(b) * D + i] = __bfloat162float(e[i]);
}

// X[b][:] = bf16(H[b] * rsqrt(mean(H[b]^2) + eps) * g)   (model.py:94-98)
// One CTA (256 threads) per row; fixed-order reduction.
__global__ void rmsnorm_rows_kernel(const float* __restrict__ H, const float* __restrict__ g, int D, float eps,
                                    __nv_bfloat16* __restrict__ X, int ldx) {
  __shared__ float red[8];
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* h = H + static_cast<size_t>(b) * D;
  float ss = 0.f;
  for (int i = t; i < D; i += 256) ss = fmaf(h[i], h[i], ss);
  ss = warp_sum(ss);
  if (lane == 0) red[warp] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int w = 0; w < 8; ++w) tot += red[w];
  const float r = rsqrtf(tot / static_cast<float>(D) + eps);
  for (int i = t; i < D; i += 256)
    X[static_cast<size_t>(b) * ldx + i] = __float2bfloat16_rn(h[i] * r * __ldg(g + i));
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
};

__device__ __forceinline__ size_t page_row(const PagedAttnArgs& a, int blk, int kv, int g, int slot) {
  return ((((static_cast<size_t>(a.layer) * a.num_blocks + blk) * 2 + kv) * a.n_kv + g) * kPageTokens + slot) * 64;
}

// grid (B, n_kv), block 32 * (n_heads / n_kv): warp w serves query head
// g * GQA + w; the K/V pages of kv head g are read once per CTA (L1 shared).
// GQA <= 4 (the shared buffers hold four query heads).
__global__ void __launch_bounds__(128) paged_attn_kernel(const __grid_constant__ PagedAttnArgs a) {
  __shared__ float sq[4][64];
  __shared__ float skn[64], svn[64];
  __shared__ float sprob[4][32];
  const int b = blockIdx.x, g = blockIdx.y, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int GQA = a.n_heads / a.n_kv;
  const int h = g * GQA + warp;
  const int p = a.pos[b];
  const int qkvd = (a.n_heads + 2 * a.n_kv) * 64;
  __nv_bfloat16* o = a.out + static_cast<size_t>(b) * a.ldo + h * 64;
  if (p < 0 || p >= a.ctx) {  // inactive (or invalid) sequence: no cache write
    reinterpret_cast<__nv_bfloat162*>(o)[lane] = __floats2bfloat162_rn(0.f, 0.f);
    return;
  }
  const float* row = a.qkv + static_cast<size_t>(b) * qkvd;
  const float c = a.rcos[static_cast<size_t>(p) * 32 + lane], s = a.rsin[static_cast<size_t>(p) * 32 + lane];
  {  // RoPE (rotate-half, model.py:110-117); q pre-scaled by 1/sqrt(64) (exact)
    const float* q = row + h * 64;
    const float lo = q[lane], hi = q[lane + 32];
    sq[warp][lane] = (lo * c - hi * s) * 0.125f;
    sq[warp][lane + 32] = (lo * s + hi * c) * 0.125f;
    if (warp == 0) {
      const float* k = row + a.n_heads * 64 + g * 64;
      const float klo = k[lane], khi = k[lane + 32];
      skn[lane] = klo * c - khi * s;
      skn[lane + 32] = klo * s + khi * c;
      const float* v = row + (a.n_heads + a.n_kv) * 64 + g * 64;
      svn[lane] = v[lane];
      svn[lane + 32] = v[lane + 32];
    }
  }
  __syncthreads();
  const int* tb = a.table + static_cast<size_t>(b) * a.bps;
  // every block this step touches must exist (checked by every warp: uniform)
  bool bad = p / kPageTokens >= a.bps;
  for (int i = lane; !bad && i <= p / kPageTokens; i += 32) bad = tb[i] < 0 || tb[i] >= a.num_blocks;
  if (__any_sync(0xffffffffu, bad)) {
    if (threadIdx.x == 0) atomicCAS(a.status, 0u, 0x203u);
    reinterpret_cast<__nv_bfloat162*>(o)[lane] = __floats2bfloat162_rn(0.f, 0.f);
    return;
  }
  if (warp == 0) {  // append this position's K (post-RoPE) / V, bf16
    const int blk = tb[p / kPageTokens], slot = p % kPageTokens;
    reinterpret_cast<__nv_bfloat162*>(a.pool + page_row(a, blk, 0, g, slot))[lane] =
        __floats2bfloat162_rn(skn[2 * lane], skn[2 * lane + 1]);
    reinterpret_cast<__nv_bfloat162*>(a.pool + page_row(a, blk, 1, g, slot))[lane] =
        __floats2bfloat162_rn(svn[2 * lane], svn[2 * lane + 1]);
  }
  // attention over positions 0..p: lane-per-position QK, lane-per-dim PV
  float m = -INFINITY, l = 0.f, o0 = 0.f, o1 = 0.f;
  for (int base = 0; base <= p; base += 32) {
    const int pp = base + lane;
    float sc = -INFINITY;
    if (pp < p) {
      const uint4* kr = reinterpret_cast<const uint4*>(a.pool + page_row(a, tb[pp / kPageTokens], 0, g, pp % kPageTokens));
      float d = 0.f;
#pragma unroll
      for (int cc = 0; cc < 8; ++cc) {
        const uint4 w = __ldg(kr + cc);
        const float* qq = sq[warp] + cc * 8;
        d = fmaf(qq[0], bf16_lo(w.x), d); d = fmaf(qq[1], bf16_hi(w.x), d);
        d = fmaf(qq[2], bf16_lo(w.y), d); d = fmaf(qq[3], bf16_hi(w.y), d);
        d = fmaf(qq[4], bf16_lo(w.z), d); d = fmaf(qq[5], bf16_hi(w.z), d);
        d = fmaf(qq[6], bf16_lo(w.w), d); d = fmaf(qq[7], bf16_hi(w.w), d);
      }
      sc = d;
    } else if (pp == p) {
      float d = 0.f;
#pragma unroll 8
      for (int k = 0; k < 64; ++k) d = fmaf(sq[warp][k], skn[k], d);
      sc = d;
    }
    float mx = sc;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float mn = fmaxf(m, mx);
    const float pe = pp <= p ? __expf(sc - mn) : 0.f;
    float ps = pe;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
    const float alpha = m == -INFINITY ? 0.f : __expf(m - mn);
    sprob[warp][lane] = pe;
    __syncwarp();
    float a0 = 0.f, a1 = 0.f;
    const int n = min(32, p + 1 - base);
    for (int i = 0; i < n; ++i) {
      const int pv = base + i;
      const float pi = sprob[warp][i];
      float v0, v1;
      if (pv == p) {
        v0 = svn[2 * lane];
        v1 = svn[2 * lane + 1];
      } else {
        const uint32_t vw = __ldg(reinterpret_cast<const unsigned int*>(
                                      a.pool + page_row(a, tb[pv / kPageTokens], 1, g, pv % kPageTokens)) + lane);
        v0 = bf16_lo(vw);
        v1 = bf16_hi(vw);
      }
      a0 = fmaf(pi, v0, a0);
      a1 = fmaf(pi, v1, a1);
    }
    __syncwarp();
    l = fmaf(l, alpha, ps);
    o0 = fmaf(o0, alpha, a0);
    o1 = fmaf(o1, alpha, a1);
    m = mn;
  }
  const float inv = 1.0f / fmaxf(l, 1e-10f);
  reinterpret_cast<__nv_bfloat162*>(o)[lane] = __floats2bfloat162_rn(o0 * inv, o1 * inv);
}

// next[b] = first index of the maximum of logits[b][0..V)  (one CTA per row)
__global__ void argmax_rows_kernel(const float* __restrict__ logits, int V, int ldl, int32_t* __restrict__ next) {
  __shared__ float rv[32];
  __shared__ int ri[32];
  const int b = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
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
