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

// H[b][:] = f32(emb[tok[b]]);  layer 0's folded RMSNorm input (model.py:94-98):
// X[b][:] = bf16(H[b] * g) and the row's sum of squares in ss[0 * ss_ld + b]
// (the other ss_tiles - 1 partials zero; the QKV projection applies
// rsqrt(mean + eps)).  One CTA (256 threads) per row; fixed-order reduction.
__global__ void embed_rows_kernel(const __nv_bfloat16* __restrict__ emb, const int32_t* __restrict__ tok,
                                  int vocab, int D, const float* __restrict__ g, float* __restrict__ H,
                                  __nv_bfloat16* __restrict__ X, float* __restrict__ ss, int ss_ld, int ss_tiles,
                                  uint32_t* status) {
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
  float q = 0.f;
  for (int i = t; i < D; i += 256) {
    const float v = __bfloat162float(e[i]);
    h[i] = v;
    X[static_cast<size_t>(b) * D + i] = __float2bfloat16_rn(v * __ldg(g + i));
    q = fmaf(v, v, q);
  }
  q = warp_sum(q);
  if (lane == 0) red[warp] = q;
  __syncthreads();
  if (t < ss_tiles) {
    float tot = 0.f;
    if (t == 0)
#pragma unroll
      for (int w = 0; w < 8; ++w) tot += red[w];
    ss[static_cast<size_t>(t) * ss_ld + b] = tot;
  }
}

struct PagedAttnArgs {
  const float* qkv;            // [B][(H+2KVH)*64] f32 (pre-RoPE q, k; v)
  const int32_t* pos;          // [B]
  __nv_bfloat16* pool;         // paged KV pool
  const int32_t* table;        // row b's entries at table + b * table_ld
  int bps, num_blocks, layer, n_heads, n_kv, ctx;
  int table_ld;                // bps (decode: one table row per sequence) or 0 (prefill: rows share row 0)
  const float* rcos;           // [ctx][32]
  const float* rsin;
  __nv_bfloat16* out;          // [B][ldo] bf16: head h at columns h*64..
  int ldo;
  uint32_t* status;            // set when a block-table entry is out of range
  int cpc;                     // units per (row, kv head) (1, 2 or 4), each an even share of the row's pages
  // Cache addressing: table != nullptr -> the paged pool above; table ==
  // nullptr -> one sequence's contiguous cache in the reference layout
  // [layer][K|V][kv_head][ctx][64].  In a prefill every row of the launch is a
  // position of one sequence (table_ld = 0 with a paged pool).
  bool append;                 // the CTA holding a row's position writes its K/V (else done before)
  // diagnostics: global-timer stamps [unit][8] (units >= trace_units skipped), or nullptr
  uint64_t* trace;
  int trace_units;
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
  const int32_t* tb = a.table ? a.table + static_cast<size_t>(b) * a.table_ld : nullptr;
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
