// attn_paged.cuh — decode attention over a paged (or contiguous) KV cache on
// warp-level tensor-core MMAs (sm_100a).
//
// Every warp is an independent attention unit (row b, kv head g, split x):
// it takes an even share x of the 16-position pages 0 .. pos[b]/16 of row b
// (split by the row's actual length, so a launch captured once serves every
// position) and runs its own online softmax over them for the GQA query heads
// of g.  The splits (1, 2 or 4) units of a (row, kv head) are consecutive
// warps of one CTA of W = max(2, splits) warps.
//
//   * page loads: each lane copies 4 + 4 16-byte pieces of the page's K and V
//     rows (2 KB each, contiguous in the pool) with `cp.async` into a
//     kPaStages-deep ring private to the warp (rows padded to 144 B, so the
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
// A unit that covers its whole row writes the output directly; when a row is
// split, each unit leaves its (m, l, o) partial in its own shared memory and,
// after a named barrier of the row's warps, the first of them merges the
// partials in split order.  Every reduction has a fixed order: results are
// bitwise reproducible.  The unit holding position
// pos[b] uses the new K (post-RoPE) / V rounded to bf16 (the cached values)
// and, in append mode, writes them to the cache.  Math: model.py:
// 100-131 (rotate-half RoPE, causal softmax over 0..p, GQA sharing).
#pragma once

#include <cuda_bf16.h>

#include "batched.cuh"
#include "tc_ptx.cuh"

namespace b2d {

constexpr int kPaStages = 6;    // pages in each warp's ring (consumed two at a time)
constexpr int kPaStagesShallow = 4;  // the ring when units far outnumber warp slots (more warps per SM)
constexpr int kPaStagesSplit = 2;    // the ring of rows split in two so that their units fit one wave
constexpr int kPaPitch = 72;    // bf16 per staged row: 144 B
constexpr int kPaStageElems = 2 * kPageTokens * kPaPitch;  // K rows then V rows
constexpr int kPaMaxSplits = 4; // units per (row, kv head)
constexpr int kPaWarpSmem = kPaStages * kPaStageElems * 2 + 256;  // ring + the new K / V row (bytes)
// TMA page path (paged pool): a page's K and V rows land as two 2 KB tensor
// copies with the 128-byte swizzle (16-byte chunk c of row r at chunk
// c ^ (r % 8)), so the ldmatrix row reads are conflict-free without padding.
constexpr int kPaPageBytes = 2 * kPageTokens * 128;                  // K then V, 4 KB
constexpr int kPaWarpSmemTma = kPaStages * kPaPageBytes + 1024;      // ring + new K/V row + mbarriers (1024-aligned)
constexpr uint64_t kPaWaitNs = 200000000ull;                          // bound on every page wait
static_assert(kPaStages * kPaPageBytes + 256 + 8 * kPaStages <= kPaWarpSmemTma, "TMA ring layout");
static_assert(kPaWarpSmemTma % 1024 == 0, "every warp's ring starts 1024-byte aligned");
// Dynamic shared memory of a CTA of W warps.
// Bytes per warp for a ring of `stages` pages.
constexpr __host__ __device__ int pa_warp_smem(bool tma, int stages) {
  return tma ? stages * kPaPageBytes + 1024 : stages * kPaStageElems * 2 + 256;
}
constexpr __host__ __device__ int pa_smem_bytes(int w, bool tma, int stages = kPaStages) {
  return tma ? w * pa_warp_smem(true, stages) + 1024 : w * pa_warp_smem(false, stages);
}
static_assert(pa_warp_smem(true, kPaStages) == kPaWarpSmemTma && pa_warp_smem(false, kPaStages) == kPaWarpSmem,
              "ring sizes");
static_assert(pa_warp_smem(true, kPaStagesShallow) % 1024 == 0 && pa_warp_smem(true, kPaStagesSplit) % 1024 == 0,
              "every warp's ring starts 1024-byte aligned");
// Byte offset of 16-byte chunk c of row r inside a swizzled 16-row tile.
__device__ __forceinline__ uint32_t sw128(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}
// warps per CTA for a split count (a row's units share a CTA)
constexpr __host__ __device__ int pa_warps(int splits) { return splits > 2 ? splits : 2; }

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

// First element of page `pg`'s K (kv = 0) or V (kv = 1) rows: 16 rows of 64
// (paged pool: physical block `blk`; contiguous cache: blk unused).
__device__ __forceinline__ const __nv_bfloat16* page_rows(const PagedAttnArgs& a, int blk, int pg, int kv, int g) {
  if (a.table == nullptr)
    return a.pool + ((((static_cast<size_t>(a.layer) * 2 + kv) * a.n_kv + g) * a.ctx) + pg * kPageTokens) * 64;
  return a.pool + (((static_cast<size_t>(a.layer) * a.num_blocks + blk) * 2 + kv) * a.n_kv + g) *
                      (kPageTokens * 64);
}

// grid ceil(rows * n_kv * splits / W), W * 32 threads, pa_smem_bytes(W, TMA)
// bytes of dynamic shared memory; a.cpc = splits (1, 2 or 4), W =
// pa_warps(splits).  Unit u = blockIdx.x * W + warp is (b, g, x) with u =
// (b * n_kv + g) * splits + x.  TMA = true needs a paged pool (a.table) and
// kvmap: the pool as rows of 64 bf16 (128 B), boxes of 16 rows, 128-byte
// swizzle; otherwise kvmap is unused and pages arrive by per-lane cp.async.
template <int W, bool TMA, int STAGES = kPaStages>
__global__ void __launch_bounds__(32 * W) paged_attn_mma_kernel(const __grid_constant__ CUtensorMap kvmap,
                                                                const __grid_constant__ PagedAttnArgs a, int n_rows) {
  extern __shared__ __align__(16) uint8_t pa_smem_raw[];
  constexpr int WS = pa_warp_smem(TMA, STAGES);  // bytes per warp
  uint8_t* pa_smem = TMA ? reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pa_smem_raw) + 1023) & ~uintptr_t(1023))
                         : pa_smem_raw;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gid = lane >> 2, tig = lane & 3;
  const int splits = a.cpc;
  const int u = blockIdx.x * W + warp;
  if (u >= n_rows * a.n_kv * splits) return;
  const int x = u % splits, g = (u / splits) % a.n_kv, b = u / (splits * a.n_kv);
  // diagnostics: 0 entry, 1 loads issued, 2 past the programmatic wait, 3 query ready,
  // 4 first page done, 5 pages done, 6 result / partial written, 7 merged
  uint64_t* trace = a.trace != nullptr && u < a.trace_units ? a.trace + static_cast<size_t>(u) * 8 : nullptr;
  auto stamp = [&](int slot) {
    if (trace != nullptr && lane == 0) trace[slot] = globaltimer_ns();
  };
  stamp(0);
  __nv_bfloat16* ring = reinterpret_cast<__nv_bfloat16*>(pa_smem + warp * WS);
  // the new position's K / V (bf16, as cached) after the ring
  __nv_bfloat16* skn = TMA ? reinterpret_cast<__nv_bfloat16*>(pa_smem + warp * WS + STAGES * kPaPageBytes)
                           : ring + STAGES * kPaStageElems;
  __nv_bfloat16* svn = skn + 64;
  uint64_t* pbar = reinterpret_cast<uint64_t*>(skn + 128);  // TMA: one mbarrier per ring slot
  if (TMA && lane == 0) {
    for (int i = 0; i < STAGES; ++i) mbar_init(&pbar[i], 1);
    fence_mbar_init();
    tma_prefetch_desc(&kvmap);
  }
  __syncwarp();
  const int GQA = a.n_heads / a.n_kv;
  const bool early = a.append;  // decode: the cache pages do not depend on the waited-for kernel
  if (!early) {
    pdl_wait();
    pdl_launch();
  }
  const int32_t* tb = a.table ? a.table + static_cast<size_t>(b) * a.table_ld : nullptr;
  // The row's first 32 block-table entries, read alongside the position (lane i: page i).
  const int tbl = tb != nullptr && lane < a.bps ? __ldg(tb + lane) : 0;
  const int p = a.pos[b];
  if (p < 0 || p >= a.ctx) {  // idle row: no cache write, zero output
    if (early) {
      pdl_wait();
      pdl_launch();
    }
    if (x == 0)
      for (int i = lane; i < GQA * 32; i += 32)
        reinterpret_cast<__nv_bfloat162*>(a.out + static_cast<size_t>(b) * a.ldo + g * GQA * 64)[i] =
            __floats2bfloat162_rn(0.f, 0.f);
    return;
  }
  const int npg = p / kPageTokens + 1;
  const int ppu = (npg + splits - 1) / splits;  // pages per unit
  const int pg_lo = min(x * ppu, npg);          // a unit past the row's pages has none (it still merges)
  const int pg_hi = min(pg_lo + ppu, npg);
  const bool owner = pg_lo < npg && pg_hi == npg;  // this unit's last page holds position p
  bool bad = tb != nullptr && npg > a.bps;
  if (tb != nullptr && !bad) {  // every page of the unit must exist
    if (lane >= pg_lo && lane < pg_hi) bad = tbl < 0 || tbl >= a.num_blocks;
    for (int i = max(pg_lo, 32) + lane; i < pg_hi; i += 32) {
      const int e = tb[i];
      bad = bad || e < 0 || e >= a.num_blocks;
    }
  }
  bad = __any_sync(0xffffffffu, bad);

  // ---- page ring ----
  const int nw = bad ? 0 : pg_hi - pg_lo;
  const int rows_max = a.table == nullptr ? a.ctx : 1 << 30;  // contiguous cache: no row past the context
  const uint64_t pol = l2_policy_evict_first();  // every K/V page is read once per step
  auto issue = [&](int k) {
    const int pg = pg_lo + k;  // (warp-uniform)
    const int blk = tb == nullptr ? 0 : pg < 32 ? __shfl_sync(0xffffffffu, tbl, pg) : tb[pg];
    if constexpr (TMA) {
      if (lane == 0) {
        const int slot = k % STAGES;
        uint8_t* dst = reinterpret_cast<uint8_t*>(ring) + slot * kPaPageBytes;
        const int rk = (((a.layer * a.num_blocks + blk) * 2) * a.n_kv + g) * kPageTokens;  // K rows (host checks the range)
        mbar_arrive_expect_tx(&pbar[slot], kPaPageBytes);
        tma_load_2d(dst, &kvmap, 0, rk, &pbar[slot], pol);
        tma_load_2d(dst + kPaPageBytes / 2, &kvmap, 0, rk + a.n_kv * kPageTokens, &pbar[slot], pol);
      }
      return;
    }
    const __nv_bfloat16* ks = page_rows(a, blk, pg, 0, g);
    const __nv_bfloat16* vs = page_rows(a, blk, pg, 1, g);
    const uint32_t dst = smem_addr(ring + (k % STAGES) * kPaStageElems);
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
  for (int k = 0; k < STAGES; ++k) {
    if (k < nw) issue(k);
    if (!TMA) cp_async_commit();
  }
  // TMA: waits for page k's copies (bounded; a timeout sets the status word and
  // the page's data are not used for anything that is written out)
  bool tma_ok = true;
  auto wait_page = [&](int k) {
    const uint32_t par = static_cast<uint32_t>(k / STAGES) & 1u;
    uint64_t* bar = &pbar[k % STAGES];
    if (mbar_test(bar, par)) return;
    const uint64_t t0 = globaltimer_ns();
    uint32_t n = 0;
    while (!mbar_test(bar, par)) {
      if ((++n & 255u) == 0 && globaltimer_ns() - t0 > kPaWaitNs) {
        if (lane == 0) atomicCAS(a.status, 0u, 0x10Cu);  // timeout | site 12 (attention pages)
        tma_ok = false;
        return;
      }
    }
  };
  // RoPE factors of position p (model constants): lane (gid, tig) needs pairs
  // 2tig, 2tig+1 and 8+2tig, 9+2tig of k-steps 0, 1; the owner's K row needs lane.
  float2 rc[2][2], rs[2][2];
#pragma unroll
  for (int s2 = 0; s2 < 2; ++s2)
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      rc[s2][h2] = *reinterpret_cast<const float2*>(a.rcos + static_cast<size_t>(p) * 32 + 16 * s2 + 8 * h2 + 2 * tig);
      rs[s2][h2] = *reinterpret_cast<const float2*>(a.rsin + static_cast<size_t>(p) * 32 + 16 * s2 + 8 * h2 + 2 * tig);
    }
  const float cs_l = a.rcos[static_cast<size_t>(p) * 32 + lane], sn_l = a.rsin[static_cast<size_t>(p) * 32 + lane];
  stamp(1);
  if (early) {
    pdl_wait();
    pdl_launch();
  }
  stamp(2);
  if (bad && lane == 0) atomicCAS(a.status, 0u, 0x203u);

  // ---- query fragments (rows gid < GQA: head g*GQA + gid; hi part rows 0..7, lo part rows 8..15) ----
  const float* row = a.qkv + static_cast<size_t>(b) * (a.n_heads + 2 * a.n_kv) * 64;
  // the new position's K / V row (owner unit), loaded beside the query so the
  // two reads of the projection's output overlap
  float nk0 = 0.f, nk1 = 0.f, nv0 = 0.f, nv1 = 0.f;
  if (owner) {
    const float* k = row + a.n_heads * 64 + g * 64;
    const float* v = row + (a.n_heads + a.n_kv) * 64 + g * 64;
    nk0 = k[lane];
    nk1 = k[lane + 32];
    nv0 = v[lane];
    nv1 = v[lane + 32];
  }
  uint32_t qa[4][4];  // [k-step][a0..a3]
  {
    float qv[4][4];   // [k-step][2tig, 2tig+1, 8+2tig, 9+2tig]
    if (gid < GQA) {
      const float* q = row + (g * GQA + gid) * 64;
#pragma unroll
      for (int s = 0; s < 4; ++s) {
        const float2 v0 = *reinterpret_cast<const float2*>(q + 16 * s + 2 * tig);
        const float2 v1 = *reinterpret_cast<const float2*>(q + 16 * s + 8 + 2 * tig);
        qv[s][0] = v0.x; qv[s][1] = v0.y; qv[s][2] = v1.x; qv[s][3] = v1.y;
      }
#pragma unroll
      for (int s = 0; s < 2; ++s) {  // rotate-half RoPE: dims d and d + 32 are k-steps s and s + 2
        const float cs[4] = {rc[s][0].x, rc[s][0].y, rc[s][1].x, rc[s][1].y};
        const float sn[4] = {rs[s][0].x, rs[s][0].y, rs[s][1].x, rs[s][1].y};
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
  if (owner) {  // the new position's K (post-RoPE) / V, bf16 as cached
    const float cs = cs_l, sn = sn_l;
    const __nv_bfloat16 k0 = __float2bfloat16_rn(nk0 * cs - nk1 * sn), k1 = __float2bfloat16_rn(nk0 * sn + nk1 * cs);
    const __nv_bfloat16 v0 = __float2bfloat16_rn(nv0), v1 = __float2bfloat16_rn(nv1);
    skn[lane] = k0;
    skn[lane + 32] = k1;
    svn[lane] = v0;
    svn[lane + 32] = v1;
    if (!bad && a.append) {
      __nv_bfloat16* kd = kv_row(a, tb, p, 0, g);
      __nv_bfloat16* vd = kv_row(a, tb, p, 1, g);
      kd[lane] = k0;
      kd[lane + 32] = k1;
      vd[lane] = v0;
      vd[lane + 32] = v1;
    }
    __syncwarp();
  }
  stamp(3);

  // ---- the unit's pages ----
  float o[8][4];  // [dim n-tile][c0..c3]: rows gid (hi) and gid + 8 (lo) of head gid
#pragma unroll
  for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m = -INFINITY, l = 0.f;
  const bool head = gid < GQA;
  // ldmatrix lane addressing: matrix mi = lane / 8, row lane % 8
  const int mi = lane >> 3, mr = lane & 7;
  static_assert(STAGES % 2 == 0, "pages are consumed in pairs");
#pragma unroll 1
  for (int k = 0; k < nw; k += 2) {  // pages k, k + 1 (when present) as one block of 32 positions
    const int pg = pg_lo + k;
    const bool two = k + 1 < nw;
    __nv_bfloat16* st0 = TMA ? reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(ring) + (k % STAGES) * kPaPageBytes)
                             : ring + (k % STAGES) * kPaStageElems;
    __nv_bfloat16* st1 = TMA ? reinterpret_cast<__nv_bfloat16*>(reinterpret_cast<uint8_t*>(ring) + ((k + 1) % STAGES) * kPaPageBytes)
                             : ring + ((k + 1) % STAGES) * kPaStageElems;
    if constexpr (TMA) {
      wait_page(k);
      if (two) wait_page(k + 1);
    } else {
      cp_async_wait<STAGES - 2>();
    }
    __syncwarp();
    if (pg == npg - 1 || (two && pg + 1 == npg - 1)) {  // the page of position p: its row from the new
      __nv_bfloat16* st = pg == npg - 1 ? st0 : st1;   // K / V, V rows past p zeroed
      const int rp = p - (npg - 1) * kPageTokens;
      if constexpr (TMA) {
        uint8_t* sbt = reinterpret_cast<uint8_t*>(st);
        if (lane < 8)
          *reinterpret_cast<uint4*>(sbt + sw128(rp, lane)) = reinterpret_cast<const uint4*>(skn)[lane];
        else if (lane < 16)
          *reinterpret_cast<uint4*>(sbt + kPaPageBytes / 2 + sw128(rp, lane - 8)) =
              reinterpret_cast<const uint4*>(svn)[lane - 8];
        for (int i = lane; i < kPageTokens * 8; i += 32) {
          const int r = i >> 3;
          if (r > rp) *reinterpret_cast<uint4*>(sbt + kPaPageBytes / 2 + r * 128 + (i & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        // these generic stores precede the slot's next tensor copy (a later page)
        fence_proxy_async_smem();
      } else {
        if (lane < 8)
          *reinterpret_cast<uint4*>(st + rp * kPaPitch + lane * 8) = reinterpret_cast<const uint4*>(skn)[lane];
        else if (lane < 16)
          *reinterpret_cast<uint4*>(st + (kPageTokens + rp) * kPaPitch + (lane - 8) * 8) =
              reinterpret_cast<const uint4*>(svn)[lane - 8];
        for (int i = lane; i < kPageTokens * 8; i += 32) {
          const int r = i >> 3;
          if (r > rp) *reinterpret_cast<uint4*>(st + (kPageTokens + r) * kPaPitch + (i & 7) * 8) = make_uint4(0, 0, 0, 0);
        }
      }
      __syncwarp();
    }
    const uint32_t sb0 = smem_addr(st0), sb1 = smem_addr(st1);
    // scores: n-tiles j (positions 8j..8j+7 of the block: page j / 2), k-steps s (dims 16s..16s+15)
    float sc[4][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
    for (int s2 = 0; s2 < 4; s2 += 2)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (j >= 2 && !two) continue;
        uint32_t b0, b1, b2, b3;  // (s2: dims +0, +8), (s2 + 1: dims +0, +8)
        const int kr = 8 * (j & 1) + mr;  // K row of the page
        ldsm_x4((j < 2 ? sb0 : sb1) + (TMA ? sw128(kr, 2 * s2 + mi) : 2u * (kr * kPaPitch + 16 * s2 + 8 * mi)), b0, b1, b2,
                b3);
        mma_bf16(sc[j], qa[s2][0], qa[s2][1], qa[s2][2], qa[s2][3], b0, b1);
        mma_bf16(sc[j], qa[s2 + 1][0], qa[s2 + 1][1], qa[s2 + 1][2], qa[s2 + 1][3], b2, b3);
      }
    // head gid's scores: block positions 8j + 2tig + e (hi + lo rows)
    float s8[8];
    const int q0 = pg * kPageTokens + 2 * tig;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const float v = sc[j][e] + sc[j][2 + e];
        s8[2 * j + e] = head && (j < 2 || two) && q0 + 8 * j + e <= p ? v : -INFINITY;
      }
    float mx = s8[0];
#pragma unroll
    for (int e = 1; e < 8; ++e) mx = fmaxf(mx, s8[e]);
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float mn = fmaxf(m, mx);  // finite for heads: position pg*16 <= p is in every block
    const float alpha = m == -INFINITY ? 0.f : __expf(m - mn);
    float pr[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) pr[e] = s8[e] == -INFINITY ? 0.f : __expf(s8[e] - mn);
    m = head ? mn : -INFINITY;
    l = fmaf(l, alpha, ((pr[0] + pr[1]) + (pr[2] + pr[3])) + ((pr[4] + pr[5]) + (pr[6] + pr[7])));
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      o[j][0] *= alpha; o[j][1] *= alpha; o[j][2] *= alpha; o[j][3] *= alpha;
    }
    // P.V per page: A rows gid = P hi, gid + 8 = P lo; k = the page's positions; V rows (ldmatrix.trans)
#pragma unroll
    for (int pp = 0; pp < 2; ++pp) {
      if (pp == 1 && !two) break;
      uint32_t pa0, pa1, pa2, pa3;
      split_bf2(pr[4 * pp + 0], pr[4 * pp + 1], pa0, pa1);
      split_bf2(pr[4 * pp + 2], pr[4 * pp + 3], pa2, pa3);
      const uint32_t sb = pp == 0 ? sb0 : sb1;
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        uint32_t b0, b1, b2, b3;  // (tile j: rows 0-7, 8-15), (tile j+1: rows 0-7, 8-15)
        const int vr = (mi & 1) * 8 + mr;  // V row of the page
        ldsm_x4_t(sb + (TMA ? kPaPageBytes / 2 + sw128(vr, j + (mi >> 1))
                            : 2u * ((kPageTokens + vr) * kPaPitch + 8 * (j + (mi >> 1)))),
                  b0, b1, b2, b3);
        mma_bf16(o[j], pa0, pa1, pa2, pa3, b0, b1);
        mma_bf16(o[j + 1], pa0, pa1, pa2, pa3, b2, b3);
      }
    }
    __syncwarp();  // every lane's reads of these stages are done before they are refilled
    if (k + STAGES < nw) issue(k + STAGES);
    if (!TMA) cp_async_commit();
    if (k + 1 + STAGES < nw) issue(k + 1 + STAGES);
    if (!TMA) cp_async_commit();
    if (k == 0) stamp(4);
  }
  if (!TMA) cp_async_wait<0>();  // (TMA: every issued page was waited for in the loop)
  if (TMA && !tma_ok) {
    // a page wait ran out (status word set; this row's output is not meaningful):
    // wait once more, bounded, for every slot's last copy so none is in flight at
    // exit; the warp goes on to the row's barrier like the others
    for (int k = max(0, nw - STAGES); k < nw; ++k) wait_page(k);
  }
  stamp(5);
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);

  // lane (gid < GQA, tig) holds head g*GQA + gid, dims 8j + 2tig, 8j + 2tig + 1 (j < 8)
  if (splits == 1) {
    if (head) {
      const float inv = l > 0.f ? 1.0f / l : 0.f;
      __nv_bfloat162* out = reinterpret_cast<__nv_bfloat162*>(a.out + static_cast<size_t>(b) * a.ldo +
                                                             (g * GQA + gid) * 64);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        out[4 * j + tig] = __floats2bfloat162_rn((o[j][0] + o[j][2]) * inv, (o[j][1] + o[j][3]) * inv);
    }
    stamp(6);
    stamp(7);
    return;
  }
  // Partial (m, l, o) of this unit in its own (drained) ring: [head][64] o, then m[4], l[4].
  float* mine = reinterpret_cast<float*>(ring);
  if (head) {
#pragma unroll
    for (int j = 0; j < 8; ++j)
      *reinterpret_cast<float2*>(mine + gid * 64 + 8 * j + 2 * tig) = make_float2(o[j][0] + o[j][2], o[j][1] + o[j][3]);
    if (tig == 0) {
      mine[256 + gid] = m;
      mine[260 + gid] = l;
    }
  }
  stamp(6);
  // the row's warps meet: with splits > 1 they are the whole CTA (splits == W); barrier 1
  asm volatile("bar.sync 1, %0;" ::"n"(32 * W) : "memory");
  if (x == 0) {  // merge in split order: lane (hh = lane / 8, c = lane % 8) takes head hh, dims 8c .. 8c+7
    const int hh = lane >> 3, c8 = lane & 7;
    if (hh < GQA) {
      float M = -INFINITY;
      for (int j = 0; j < splits; ++j)
        M = fmaxf(M, reinterpret_cast<const float*>(pa_smem + (warp + j) * WS)[256 + hh]);
      float L = 0.f, r[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int j = 0; j < splits; ++j) {
        const float* pj = reinterpret_cast<const float*>(pa_smem + (warp + j) * WS);
        const float mj = pj[256 + hh];
        const float wgt = mj == -INFINITY ? 0.f : __expf(mj - M);
        L = fmaf(wgt, pj[260 + hh], L);
        const float4 oa = *reinterpret_cast<const float4*>(pj + hh * 64 + 8 * c8);
        const float4 ob = *reinterpret_cast<const float4*>(pj + hh * 64 + 8 * c8 + 4);
        r[0] = fmaf(wgt, oa.x, r[0]); r[1] = fmaf(wgt, oa.y, r[1]);
        r[2] = fmaf(wgt, oa.z, r[2]); r[3] = fmaf(wgt, oa.w, r[3]);
        r[4] = fmaf(wgt, ob.x, r[4]); r[5] = fmaf(wgt, ob.y, r[5]);
        r[6] = fmaf(wgt, ob.z, r[6]); r[7] = fmaf(wgt, ob.w, r[7]);
      }
      const float inv = L > 0.f ? 1.0f / L : 0.f;
      uint4 pk;
      pk.x = bf2_rn(r[0] * inv, r[1] * inv);
      pk.y = bf2_rn(r[2] * inv, r[3] * inv);
      pk.z = bf2_rn(r[4] * inv, r[5] * inv);
      pk.w = bf2_rn(r[6] * inv, r[7] * inv);
      *reinterpret_cast<uint4*>(a.out + static_cast<size_t>(b) * a.ldo + (g * GQA + hh) * 64 + 8 * c8) = pk;
    }
  }
  stamp(7);
}

}  // namespace b2d
