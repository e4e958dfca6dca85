// attn_paged.cuh — decode attention over a paged (or contiguous) KV cache on
// warp-level tensor-core MMAs (sm_100a).
//
// grid (splits, n_kv, rows), 4 warps.  CTA (x, g, b) takes an even share of
// the 16-position pages 0 .. pos[b]/16 of row b (split by the row's actual
// length, so a launch captured once serves every position), its warps take
// the CTA's pages round-robin, and every warp runs its own online softmax:
//
//   * page loads: each lane copies 4 + 4 16-byte pieces of the page's K and V
//     rows (2 KB each, contiguous in the pool) with `cp.async` into a
//     two-stage ring private to the warp (rows padded to 144 B, so the
//     `ldmatrix` row reads below are conflict-free).  In decode (append) mode
//     the first pages are requested before the programmatic wait: they only
//     depend on earlier steps, not on the QKV projection being waited for.
//   * scores: `mma.m16n8k16` bf16 -> f32 with the GQA query heads as rows
//     0..3 and the low-order bf16 part of each query as rows 8..11 (q = hi +
//     lo, both bf16: the product is exact to ~2^-17), the page's 16 K rows as
//     two n-tiles (`ldmatrix`);  a lane's four scores are positions 2t, 2t+1,
//     2t+8, 2t+9 of head lane/4, which are exactly its A-fragment entries for
//     the P.V product, so the probabilities never leave registers.
//   * P.V: `mma.m16n8k16` with P = hi + lo bf16 again (rows 0..3 / 8..11) and
//     the V rows as B (`ldmatrix.trans`), 8 n-tiles of dimensions.
//
// The warps' (m, l, o) are merged in warp order in shared memory; when a row
// spans several CTAs each writes its (m, l, o) partial and the last CTA to
// take the (row, kv head) ticket merges them in CTA order.  Every reduction
// has a fixed order: results are bitwise reproducible.  The CTA holding
// position pos[b] uses the new K (post-RoPE) / V rounded to bf16 (the cached
// values) and, in append mode, writes them to the cache.  Math: model.py:
// 100-131 (rotate-half RoPE, causal softmax over 0..p, GQA sharing).
#pragma once

#include <cuda_bf16.h>

#include "batched.cuh"

namespace b2d {

constexpr int kPaWarps = 4;     // warps per CTA
constexpr int kPaStages = 2;    // pages in each warp's ring
constexpr int kPaPitch = 72;    // bf16 per staged row: 144 B
constexpr int kPaStageElems = 2 * kPageTokens * kPaPitch;  // K rows then V rows
constexpr int kPaMaxSplits = 8; // CTAs per (row, kv head); <= the partial buffer's chunks

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// d += a * b, m16n8k16, bf16 inputs, f32 accumulators.
__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t bf2_rn(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}
// x = hi + lo with hi = bf16(x), lo = bf16(x - hi): packed pairs (x0, x1).
__device__ __forceinline__ void split_bf2(float x0, float x1, uint32_t& hi, uint32_t& lo) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(x0, x1);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = bf2_rn(x0 - __low2float(h), x1 - __high2float(h));
}

// First element of page `pg`'s K (kv = 0) or V (kv = 1) rows: 16 rows of 64.
__device__ __forceinline__ const __nv_bfloat16* page_rows(const PagedAttnArgs& a, const int32_t* tb, int pg,
                                                          int kv, int g) {
  if (a.table == nullptr)
    return a.pool + ((((static_cast<size_t>(a.layer) * 2 + kv) * a.n_kv + g) * a.ctx) + pg * kPageTokens) * 64;
  return a.pool + (((static_cast<size_t>(a.layer) * a.num_blocks + tb[pg]) * 2 + kv) * a.n_kv + g) *
                      (kPageTokens * 64);
}

__global__ void __launch_bounds__(32 * kPaWarps, 5) paged_attn_mma_kernel(const __grid_constant__ PagedAttnArgs a) {
  __shared__ __align__(16) __nv_bfloat16 stage[kPaWarps][kPaStages][kPaStageElems];
  __shared__ __align__(16) __nv_bfloat16 skn[64], svn[64];  // the new position's K / V (bf16, as cached)
  __shared__ float wm[kPaWarps][4], wl[kPaWarps][4];
  __shared__ uint32_t s_last;
  const int x = blockIdx.x, g = blockIdx.y, b = blockIdx.z;
  const int t = threadIdx.x, warp = t >> 5, lane = t & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int GQA = a.n_heads / a.n_kv;
  const bool early = a.append;  // decode: the cache pages do not depend on the waited-for kernel
  if (!early) {
    pdl_wait();
    pdl_launch();
  }
  const int p = a.pos[b];
  if (p < 0 || p >= a.ctx) {  // idle row: no cache write, zero output
    if (early) {
      pdl_wait();
      pdl_launch();
    }
    if (x == 0 && warp < GQA)
      reinterpret_cast<__nv_bfloat162*>(a.out + static_cast<size_t>(b) * a.ldo + (g * GQA + warp) * 64)[lane] =
          __floats2bfloat162_rn(0.f, 0.f);
    return;
  }
  const int npg = p / kPageTokens + 1;
  const int ppc = (npg + a.cpc - 1) / a.cpc;  // pages per CTA (a.cpc = splits)
  const int pg_lo = x * ppc;
  if (pg_lo >= npg) return;  // no pages for this CTA: no ticket either
  const int pg_hi = min(pg_lo + ppc, npg);
  const int ncta = (npg + ppc - 1) / ppc;  // CTAs sharing this (row, kv head)
  const bool owner = pg_hi == npg;
  const int32_t* tb = a.table ? a.table + static_cast<size_t>(b) * a.bps : nullptr;
  bool bad = tb != nullptr && npg > a.bps;
  for (int i = pg_lo + t; tb != nullptr && !bad && i < pg_hi; i += 32 * kPaWarps) {
    const int e = tb[i];
    bad = e < 0 || e >= a.num_blocks;
  }
  bad = __syncthreads_or(bad);

  // ---- this warp's pages: pg_lo + warp + kPaWarps * k, k < nw ----
  const int nw = bad ? 0 : (pg_hi - pg_lo - warp + kPaWarps - 1) / kPaWarps;
  const int rows_max = a.table == nullptr ? a.ctx : 1 << 30;  // contiguous cache: no row past the context
  auto issue = [&](int k) {
    const int pg = pg_lo + warp + kPaWarps * k;
    const __nv_bfloat16* ks = page_rows(a, tb, pg, 0, g);
    const __nv_bfloat16* vs = page_rows(a, tb, pg, 1, g);
    const uint32_t dst = smem_addr(&stage[warp][k % kPaStages][0]);
#pragma unroll
    for (int r = 0; r < 4; ++r) {
      const int i = lane + 32 * r, row = i >> 3, c16 = i & 7;
      if (pg * kPageTokens + row < rows_max) {
        cp_async16(dst + 2u * (row * kPaPitch + c16 * 8), ks + i * 8);
        cp_async16(dst + 2u * ((kPageTokens + row) * kPaPitch + c16 * 8), vs + i * 8);
      }
    }
  };
#pragma unroll
  for (int k = 0; k < kPaStages; ++k) {
    if (k < nw) issue(k);
    cp_async_commit();
  }
  if (early) {
    pdl_wait();
    pdl_launch();
  }
  if (bad && t == 0) atomicCAS(a.status, 0u, 0x203u);

  // ---- query fragments (rows gid < GQA: head g*GQA + gid; hi part rows 0..7, lo part rows 8..15) ----
  const float* row = a.qkv + static_cast<size_t>(b) * (a.n_heads + 2 * a.n_kv) * 64;
  uint32_t qa[4][4];  // [k-step][a0..a3]
  {
    float qv[4][4];   // [k-step][2tig, 2tig+1, 8+2tig, 9+2tig]
    if (gid < GQA) {
      const float* q = row + (g * GQA + gid) * 64;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const float2 u = *reinterpret_cast<const float2*>(q + 16 * s + 2 * tig);
        const float2 w = *reinterpret_cast<const float2*>(q + 16 * s + 8 + 2 * tig);
        qv[s][0] = u.x; qv[s][1] = u.y; qv[s][2] = w.x; qv[s][3] = w.y;
      }
#pragma unroll
      for (int s = 0; s < 2; ++s) {  // rotate-half RoPE: dims d and d + 32 are k-steps s and s + 2
        const float2 c0 = *reinterpret_cast<const float2*>(a.rcos + static_cast<size_t>(p) * 32 + 16 * s + 2 * tig);
        const float2 c1 = *reinterpret_cast<const float2*>(a.rcos + static_cast<size_t>(p) * 32 + 16 * s + 8 + 2 * tig);
        const float2 s0 = *reinterpret_cast<const float2*>(a.rsin + static_cast<size_t>(p) * 32 + 16 * s + 2 * tig);
        const float2 s1 = *reinterpret_cast<const float2*>(a.rsin + static_cast<size_t>(p) * 32 + 16 * s + 8 + 2 * tig);
        const float cs[4] = {c0.x, c0.y, c1.x, c1.y}, sn[4] = {s0.x, s0.y, s1.x, s1.y};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = qv[s][e], hi = qv[s + 2][e];
          qv[s][e] = (lo * cs[e] - hi * sn[e]) * 0.125f;  // pre-scaled by 1/sqrt(64) (exact)
          qv[s + 2][e] = (lo * sn[e] + hi * cs[e]) * 0.125f;
        }
      }
    } else {
#pragma unroll
      for (int s = 0; s < 4; ++s) qv[s][0] = qv[s][1] = qv[s][2] = qv[s][3] = 0.f;
    }
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      split_bf2(qv[s][0], qv[s][1], qa[s][0], qa[s][1]);
      split_bf2(qv[s][2], qv[s][3], qa[s][2], qa[s][3]);
    }
  }
  if (owner && warp == 0) {  // the new position's K (post-RoPE) / V, bf16 as cached
    const float cs = a.rcos[static_cast<size_t>(p) * 32 + lane], sn = a.rsin[static_cast<size_t>(p) * 32 + lane];
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
  __syncthreads();  // skn / svn ready

  // ---- the warp's pages ----
  float o[8][4];  // [dim n-tile][c0..c3]: rows gid (hi) and gid + 8 (lo) of head gid
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m = -INFINITY, l = 0.f;
  const bool head = gid < GQA;
  // ldmatrix lane addressing: matrix mi = lane / 8, row lane % 8
  const int mi = lane >> 3, mr = lane & 7;
#pragma unroll 1
  for (int k = 0; k < nw; ++k) {
    const int pg = pg_lo + warp + kPaWarps * k;
    __nv_bfloat16* st = &stage[warp][k % kPaStages][0];
    cp_async_wait<kPaStages - 1>();
    __syncwarp();
    if (pg == npg - 1) {  // the page of position p: its row from the new K / V, V rows past p zeroed
      const int rp = p - pg * kPageTokens;
      if (lane < 8)
        *reinterpret_cast<uint4*>(st + rp * kPaPitch + lane * 8) = reinterpret_cast<const uint4*>(skn)[lane];
      else if (lane < 16)
        *reinterpret_cast<uint4*>(st + (kPageTokens + rp) * kPaPitch + (lane - 8) * 8) =
            reinterpret_cast<const uint4*>(svn)[lane - 8];
      for (int i = lane; i < kPageTokens * 8; i += 32) {
        const int r = i >> 3;
        if (r > rp) *reinterpret_cast<uint4*>(st + (kPageTokens + r) * kPaPitch + (i & 7) * 8) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    const uint32_t sb = smem_addr(st);
    // scores: n-tiles j (positions 8j..8j+7), k-steps s (dims 16s..16s+15)
    float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int s2 = 0; s2 < 4; s2 += 2) {
        uint32_t b0, b1, b2, b3;  // (s2: dims +0, +8), (s2 + 1: dims +0, +8)
        ldsm_x4(sb + 2u * ((8 * j + mr) * kPaPitch + 16 * s2 + 8 * mi), b0, b1, b2, b3);
        mma_bf16(sc[j], qa[s2][0], qa[s2][1], qa[s2][2], qa[s2][3], b0, b1);
        mma_bf16(sc[j], qa[s2 + 1][0], qa[s2 + 1][1], qa[s2 + 1][2], qa[s2 + 1][3], b2, b3);
      }
    // head gid's scores at positions 2tig, 2tig+1 (j = 0) and 8+2tig, 9+2tig (j = 1): hi + lo rows
    float s4[4];
    const int q0 = pg * kPageTokens + 2 * tig;
#pragma unroll
    for (int j = 0; j < 2; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float v = sc[j][e] + sc[j][2 + e];
        s4[2 * j + e] = head && q0 + 8 * j + e <= p ? v : -INFINITY;
      }
    float mx = fmaxf(fmaxf(s4[0], s4[1]), fmaxf(s4[2], s4[3]));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m, mx);  // finite for heads: position pg*16 <= p is in every page
    const float alpha = m == -INFINITY ? 0.f : __expf(m - mn);
    float pr[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) pr[e] = s4[e] == -INFINITY ? 0.f : __expf(s4[e] - mn);
    m = head ? mn : -INFINITY;
    l = fmaf(l, alpha, (pr[0] + pr[1]) + (pr[2] + pr[3]));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= alpha; o[j][1] *= alpha; o[j][2] *= alpha; o[j][3] *= alpha;
    }
    uint32_t pa0, pa1, pa2, pa3;  // A: rows gid = P hi, gid + 8 = P lo; k = positions 2tig.. / 8+2tig..
    split_bf2(pr[0], pr[1], pa0, pa1);
    split_bf2(pr[2], pr[3], pa2, pa3);
    // P.V: n-tiles of 8 dimensions; V rows = k (ldmatrix.trans)
#pragma unroll
    for (int j = 0; j < 8; j += 2) {
      uint32_t b0, b1, b2, b3;  // (tile j: rows 0-7, 8-15), (tile j+1: rows 0-7, 8-15)
      ldsm_x4_t(sb + 2u * ((kPageTokens + (mi & 1) * 8 + mr) * kPaPitch + 8 * (j + (mi >> 1))), b0, b1, b2, b3);
      mma_bf16(o[j], pa0, pa1, pa2, pa3, b0, b1);
      mma_bf16(o[j + 1], pa0, pa1, pa2, pa3, b2, b3);
    }
    __syncwarp();  // every lane's reads of this stage are done before it is refilled
    if (k + kPaStages < nw) issue(k + kPaStages);
    cp_async_commit();
  }
  cp_async_wait<0>();
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);

  // ---- merge the warps in warp order (the stages are free now) ----
  __syncthreads();
  float* wo = reinterpret_cast<float*>(&stage[0][0][0]);  // [warp][4 heads][64]
  static_assert(sizeof(stage) >= kPaWarps * 4 * 64 * sizeof(float), "merge area");
  if (head) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float2*>(wo + (warp * 4 + gid) * 64 + 8 * j + 2 * tig) =
          make_float2(o[j][0] + o[j][2], o[j][1] + o[j][3]);
    if (tig == 0) {
      wm[warp][gid] = m;
      wl[warp][gid] = l;
    }
  }
  __syncthreads();
  const int h = g * GQA + warp;  // warp h < GQA merges head g*GQA + h, dims 2 lane, 2 lane + 1
  float o0 = 0.f, o1 = 0.f, M = -INFINITY, L = 0.f;
  if (warp < GQA) {
#pragma unroll
    for (int w = 0; w < kPaWarps; ++w) M = fmaxf(M, wm[w][warp]);
#pragma unroll
    for (int w = 0; w < kPaWarps; ++w) {
      const float mw = wm[w][warp];
      const float wgt = mw == -INFINITY ? 0.f : __expf(mw - M);
      const float2 v = *reinterpret_cast<const float2*>(wo + (w * 4 + warp) * 64 + 2 * lane);
      L = fmaf(wgt, wl[w][warp], L);
      o0 = fmaf(wgt, v.x, o0);
      o1 = fmaf(wgt, v.y, o1);
    }
  }
  if (ncta == 1) {
    if (warp < GQA) {
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      reinterpret_cast<__nv_bfloat162*>(a.out + static_cast<size_t>(b) * a.ldo + h * 64)[lane] =
          __floats2bfloat162_rn(o0 * inv, o1 * inv);
    }
    return;
  }
  if (warp < GQA) {
    float* part = a.part + ((static_cast<size_t>(b) * a.n_heads + h) * a.max_chunks + x) * kAttPart;
    reinterpret_cast<float2*>(part + 4)[lane] = make_float2(o0, o1);
    if (lane == 0) {
      part[0] = M;
      part[1] = L;
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
    float MM = mc;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) MM = fmaxf(MM, __shfl_xor_sync(0xffffffffu, MM, off));
    const float wl2 = mc == -INFINITY ? 0.f : __expf(mc - MM);
    float LL = wl2 * lc;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) LL += __shfl_xor_sync(0xffffffffu, LL, off);
    float r0 = 0.f, r1 = 0.f;
    for (int j = 0; j < ncta; ++j) {
      const float wgt = __shfl_sync(0xffffffffu, wl2, j);
      const float2 oc = __ldcg(reinterpret_cast<const float2*>(ph + j * kAttPart + 4) + lane);
      r0 = fmaf(wgt, oc.x, r0);
      r1 = fmaf(wgt, oc.y, r1);
    }
    const float inv = LL > 0.f ? 1.0f / LL : 0.f;
    reinterpret_cast<__nv_bfloat162*>(a.out + static_cast<size_t>(b) * a.ldo + h * 64)[lane] =
        __floats2bfloat162_rn(r0 * inv, r1 * inv);
  }
}

}  // namespace b2d
