// gemm_tc.cuh — batched-decode projections on the 5th-gen tensor cores.
//
// Y[n][m] (epilogue) = sum_k X[n][k] * W[m][k]: W is a packed weight matrix
// (output-row major, K contiguous, see include/b2d.h), X the batch of
// activation rows (bf16, K contiguous).  Both operands are K-major, staged by
// TMA with 128-byte swizzle; one thread issues tcgen05.mma (M=128 weight rows,
// N=BN batch rows, K=16) into a TMEM accumulator; the epilogue reads TMEM with
// tcgen05.ld and fuses the store: plain f32, f32 + residual, or SwiGLU of the
// interleaved gate/up rows to bf16 (the next projection's K-major input).
//
// Decode projections are short and wide (N = batch), so a weight tile alone
// would keep too few SMs busy: the K range is split over the CTAs of a
// (1, 1, ksplit) thread-block cluster.  Each CTA accumulates its K slice, the
// partial tiles meet in shared memory, and CTA r of the cluster reduces
// columns [r*BN/ks, (r+1)*BN/ks) by reading every partial through distributed
// shared memory in rank order (deterministic), then applies the epilogue.
//
// CTA = 8 warps: warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM
// allocator, all eight the epilogue (warps w and w+4 read TMEM lanes
// 32(w%4).. in alternate 32-column chunks; all 256 threads store).
// Grid = (M/128, ceil(N/BN), ksplit).  Launched with programmatic dependent
// launch: the weight tiles of the first stages are requested before waiting
// for the previous kernel (they do not depend on it).  Every wait is bounded;
// on expiry the kernel records an error word, waits (bounded) for its own
// copies in flight and leaves through the normal exit (TMEM freed).
#pragma once

#include <cuda_bf16.h>

#include "tc_ptx.cuh"

namespace b2d {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle atom of bf16
constexpr int kGemmThreads = 256;
constexpr int kGemmMaxSplit = 8;  // portable cluster size
constexpr uint64_t kGemmWaitNs = 200000000ull;  // 200 ms

enum : int { EPI_F32 = 0, EPI_RESID_F32 = 1, EPI_SWIGLU_BF16 = 2 };

struct GemmArgs {
  int M = 0, N = 0, K = 0;
  float* y = nullptr;                 // EPI_F32 / EPI_RESID_F32: [N][ldy] f32
  const float* resid = nullptr;       // EPI_RESID_F32: [N][ldy] (may equal y)
  __nv_bfloat16* ybf = nullptr;       // EPI_SWIGLU_BF16: [N][ldy] bf16, column m/2
  int ldy = 0;
  uint32_t* err = nullptr;            // status word: set (if still 0) when a wait runs out
  int ksplit = 1;                     // 1..kGemmMaxSplit, <= K/64; > 1 needs a (1,1,ksplit) cluster launch
  int n_base = 0;                     // X rows (and ss_in columns) start at this row; outputs at row 0
  // Folded RMSNorm (model.py:94-98): the next projection's input is
  // bf16(RMSNorm(h) * g) = r[n] * bf16(h * g) up to bf16 rounding, with
  // r[n] = rsqrt(mean(h[n]^2) + eps) applied to that projection's result.
  // Producer (EPI_RESID_F32 writing h): xg_out[n][m] = bf16(y * xg_gain[m])
  // and ss_out[blockIdx.x * ss_ld + n] = sum of y^2 over this tile's 128 rows.
  const float* xg_gain = nullptr;     // [M], or nullptr (no folded norm output)
  __nv_bfloat16* xg_out = nullptr;    // [N][M]
  float* ss_out = nullptr;            // [M / 128][ss_ld]
  // Consumer: column n of the result is multiplied by
  // rsqrt(sum_t ss_in[t * ss_ld + n] / ss_dim + norm_eps), t < ss_dim / 128.
  const float* ss_in = nullptr;
  int ss_dim = 0, ss_ld = 0;
  float norm_eps = 0.f;
  // diagnostics: global-timer stamps [cta][kGemmStamps] (CTAs >= trace_ctas skipped), or nullptr
  uint64_t* trace = nullptr;
  int trace_ctas = 0;
};

// Stamp slots: 0 entry, 1 prologue done, 2 producer past the programmatic
// wait, 3 first stage landed (MMA thread), 4 accumulator complete, 5 partial
// tiles exchanged (cluster barrier), 6 outputs stored, 7 exit.
constexpr int kGemmStamps = 8;
__device__ __forceinline__ void gemm_stamp(const GemmArgs& g, int slot) {
  if (g.trace == nullptr) return;
  const int cta = blockIdx.x + gridDim.x * (blockIdx.y + gridDim.y * blockIdx.z);
  if (cta < g.trace_ctas) g.trace[static_cast<size_t>(cta) * kGemmStamps + slot] = globaltimer_ns();
}

template <int BN>
struct GemmSmem {
  static constexpr int A_BYTES = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * kGemmBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int STAGES = (196608 / STAGE) < 6 ? (196608 / STAGE) : 6;
  static constexpr int BARS = STAGES * STAGE;
  static constexpr int RED_BYTES = BN * kGemmBM * 4;  // partial tile [BN][128] f32 (reuses the stages)
  static constexpr int BYTES = BARS + (2 * STAGES + 1) * 8 + 16 + 1024;  // + alignment slack
  // TMEM columns: a power of two >= 32 covering the tile's BN accumulator columns
  static constexpr uint32_t TMEM_COLS = BN <= 32 ? 32 : BN <= 64 ? 64 : BN <= 128 ? 128 : 256;
  static_assert(STAGE % 1024 == 0, "stages must keep 1024-byte alignment for the swizzle atoms");
  static_assert(RED_BYTES <= BARS, "the partial tile must fit in the stage buffers");
  static_assert(BYTES <= 227 * 1024, "shared memory per CTA");
};

// Bounded wait: gives up after kGemmWaitNs of global time, records the error.
__device__ __forceinline__ bool gemm_wait(uint64_t* bar, uint32_t parity, uint32_t* err) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t n = 0;
  while (!mbar_test(bar, parity)) {
    if ((++n & 255u) == 0 && globaltimer_ns() - t0 > kGemmWaitNs) {
      atomicCAS(err, 0u, 0x10Bu);  // timeout | site 11 (projection)
      return false;
    }
  }
  return true;
}

// Rows row..row+3 of output column n (row % 4 == 0): SwiGLU pairs (2j, 2j+1)
// lie inside the group.  `v` is final (scaled, residual added).
template <int EPI>
__device__ __forceinline__ void gemm_store4(const GemmArgs& g, float4 v, int row, int n) {
  if (EPI == EPI_SWIGLU_BF16) {
    const float a0 = v.x * __fdividef(1.0f, 1.0f + __expf(-v.x)) * v.y;  // silu(gate) * up
    const float a1 = v.z * __fdividef(1.0f, 1.0f + __expf(-v.z)) * v.w;
    *reinterpret_cast<__nv_bfloat162*>(g.ybf + static_cast<size_t>(n) * g.ldy + (row >> 1)) =
        __floats2bfloat162_rn(a0, a1);
  } else {
    *reinterpret_cast<float4*>(g.y + static_cast<size_t>(n) * g.ldy + row) = v;
  }
}

// Folded-norm producer side for one item (warp-uniform call: the 32 lanes of
// the warp hold the 32 items of one column): bf16(y * gain) and the column's
// sum of squares over the tile (butterfly order, fixed).
// `w` = xg_gain[row .. row + 3].
__device__ __forceinline__ void gemm_fold_item(const GemmArgs& g, float4 y, float4 w, int row, int n, bool live) {
  float q = 0.f;
  if (live) {
    uint2 pk;
    const __nv_bfloat162 lo = __floats2bfloat162_rn(y.x * w.x, y.y * w.y), hi = __floats2bfloat162_rn(y.z * w.z, y.w * w.w);
    pk.x = *reinterpret_cast<const uint32_t*>(&lo);
    pk.y = *reinterpret_cast<const uint32_t*>(&hi);
    *reinterpret_cast<uint2*>(g.xg_out + static_cast<size_t>(n) * g.M + row) = pk;
    q = fmaf(y.x, y.x, fmaf(y.y, y.y, fmaf(y.z, y.z, y.w * y.w)));
  }
  q = warp_sum(q);
  if (live && (threadIdx.x & 31) == 0) g.ss_out[static_cast<size_t>(blockIdx.x) * g.ss_ld + n] = q;
}

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
               const GemmArgs g) {
  using L = GemmSmem<BN>;
  constexpr int S = L::STAGES;
  extern __shared__ uint8_t gemm_smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(gemm_smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::BARS);
  uint64_t* empty = full + S;
  uint64_t* done = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ float s_rs[256];  // folded-norm consumer: scale of each tile column

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kGemmBM, n0 = blockIdx.y * BN;
  const int ks = g.ksplit;
  const int nk_all = g.K / kGemmBK;
  const int kb0 = static_cast<int>(blockIdx.z) * nk_all / ks;
  const int nk = (static_cast<int>(blockIdx.z) + 1) * nk_all / ks - kb0;

  if (threadIdx.x == 0) {
    gemm_stamp(g, 0);
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_mbar_init();
    tma_prefetch_desc(&wmap);
    tma_prefetch_desc(&xmap);
  }
  if (warp == 2) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_launch();
  if (threadIdx.x == 0) gemm_stamp(g, 1);

  int issued = 0;  // producer thread: loads requested
  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    const uint64_t pol_w = l2_policy_evict_first();
    const uint64_t pol_x = l2_policy_evict_last();
    const int pre = nk < S ? nk : S;
    for (int i = 0; i < pre; ++i) {  // weights first: independent of the previous kernel
      mbar_arrive_expect_tx(&full[i], L::STAGE);
      tma_load_2d(sm + i * L::STAGE, &wmap, (kb0 + i) * kGemmBK, m0, &full[i], pol_w);
    }
    pdl_wait();
    gemm_stamp(g, 2);
    for (int i = 0; i < pre; ++i)
      tma_load_2d(sm + i * L::STAGE + L::A_BYTES, &xmap, (kb0 + i) * kGemmBK, g.n_base + n0, &full[i], pol_x);
    issued = pre;
    for (int i = pre; i < nk; ++i) {
      const int s = i % S;
      if (!gemm_wait(&empty[s], ((i / S) - 1) & 1u, g.err)) break;
      uint8_t* a = sm + s * L::STAGE;
      mbar_arrive_expect_tx(&full[s], L::STAGE);
      tma_load_2d(a, &wmap, (kb0 + i) * kGemmBK, m0, &full[s], pol_w);
      tma_load_2d(a + L::A_BYTES, &xmap, (kb0 + i) * kGemmBK, g.n_base + n0, &full[s], pol_x);
      issued = i + 1;
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    const uint32_t idesc = idesc_bf16_f32(kGemmBM, BN);
    for (int i = 0; i < nk; ++i) {
      const int s = i % S;
      if (!gemm_wait(&full[s], (i / S) & 1u, g.err)) break;
      if (i == 0) gemm_stamp(g, 3);
      tc_fence_after();
      const uint32_t a = smem_addr(sm + s * L::STAGE);
      const uint32_t b = a + L::A_BYTES;
#pragma unroll
      for (int k = 0; k < kGemmBK / 16; ++k)
        tc_mma_bf16(tmem, sdesc_kmajor_sw128(a + 32 * k), sdesc_kmajor_sw128(b + 32 * k), idesc, i > 0 || k > 0);
      tc_commit(&empty[s]);  // stage reusable once these MMAs have read it
    }
    tc_commit(done);  // accumulator complete (or the issued part of it)
  }

  // ---- epilogue: all eight warps ----
  __syncwarp();
  pdl_wait();  // the residual and the norm statistics come from earlier kernels
  if (g.ss_in != nullptr && warp >= 2) {  // column scales (warps 2..7: idle during the main loop)
    for (int c = threadIdx.x - 64; c < BN; c += kGemmThreads - 64) {
      float rs = 1.f;
      if (n0 + c < g.N) {
        float tot = 0.f;
        for (int t = 0; t < g.ss_dim / kGemmBM; ++t)
          tot += __ldcg(g.ss_in + static_cast<size_t>(t) * g.ss_ld + g.n_base + n0 + c);
        rs = rsqrtf(tot / static_cast<float>(g.ss_dim) + g.norm_eps);
      }
      s_rs[c] = rs;
    }
  }
  // Folded-norm producer: every item of this thread covers rows m0 + 4 lane .. +3.
  const float4 gw = EPI == EPI_RESID_F32 && g.xg_out != nullptr
                        ? __ldg(reinterpret_cast<const float4*>(g.xg_gain + m0 + 4 * lane))
                        : make_float4(0.f, 0.f, 0.f, 0.f);
  const bool got = __all_sync(0xffffffffu, gemm_wait(done, 0, g.err));
  tc_fence_after();
  if (threadIdx.x == 0) gemm_stamp(g, 4);
  const int r = (warp & 3) * 32 + lane;  // accumulator row = weight row m0 + r (this warp's TMEM lanes)
  int j0 = 0, j1 = BN;  // output columns this CTA stores
  // The accumulator goes to shared memory as [BN][128] f32; the outputs are
  // then written as items of 4 consecutive rows (float4 / bf16x2 stores).
  // With a K split, the cluster's partial tiles are summed in rank order
  // through distributed shared memory and CTA `rank` stores columns
  // [rank*BN/ks, (rank+1)*BN/ks).
  float* red = reinterpret_cast<float*>(sm);  // every MMA has read its stage by now
#pragma unroll 1
  for (int c0 = (warp >> 2) * 32; c0 < BN; c0 += 64) {  // the two warp groups take alternate chunks
    float v[32];
    tmem_ld32(tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + c0, v);
#pragma unroll
    for (int j = 0; j < 32; ++j)
      if (c0 + j < BN) red[(c0 + j) * kGemmBM + r] = got ? v[j] : 0.f;
  }
  if (ks > 1) {
    cluster_sync_all();
    const int rank = static_cast<int>(cluster_ctarank());
    j0 = rank * BN / ks;
    j1 = (rank + 1) * BN / ks;
  } else {
    __syncthreads();
  }
  if (threadIdx.x == 0) gemm_stamp(g, 5);
  const int items = (j1 - j0) * (kGemmBM / 4);
  const uint32_t red_base = smem_addr(red);
  if (ks == 1) {  // the tile is local: 2 items' loads in flight per round
    // (measured, gate/up at B=256: U = 8 1.86 us, 2 1.42 us, 1 1.53 us per
    // CTA; the epilogue runs once per CTA and launch, so its code size
    // weighs against its load overlap)
    constexpr int U = 2;
#pragma unroll 1
    for (int it0 = threadIdx.x; it0 < items; it0 += U * kGemmThreads) {
      // every load of the round (tile, column scale, residual) before any store:
      // the stores go through generic pointers the loads cannot be moved past
      float4 v[U], rr[U];
      float rs[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int it = it0 + u * kGemmThreads;
        if (it < items) {
          const int j = j0 + it / (kGemmBM / 4), r4 = (it % (kGemmBM / 4)) * 4;
          v[u] = *reinterpret_cast<const float4*>(red + kGemmBM * j + r4);
          rs[u] = g.ss_in != nullptr ? s_rs[j] : 1.f;
          if (EPI == EPI_RESID_F32 && n0 + j < g.N)
            rr[u] = __ldcg(reinterpret_cast<const float4*>(g.resid + static_cast<size_t>(n0 + j) * g.ldy + m0 + r4));
        }
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int it = it0 + u * kGemmThreads;
        if (it < items) {
          const int j = j0 + it / (kGemmBM / 4), r4 = (it % (kGemmBM / 4)) * 4;
          const int n = n0 + j, rw = m0 + r4;
          const bool live = got && n < g.N && rw < g.M;
          float4 y = v[u];
          y.x *= rs[u]; y.y *= rs[u]; y.z *= rs[u]; y.w *= rs[u];
          if (EPI == EPI_RESID_F32 && live) {
            y.x += rr[u].x; y.y += rr[u].y; y.z += rr[u].z; y.w += rr[u].w;
          }
          if (live) gemm_store4<EPI>(g, y, rw, n);
          if (EPI == EPI_RESID_F32 && g.xg_out != nullptr) gemm_fold_item(g, y, gw, rw, n, live);
        }
      }
    }
  }
#pragma unroll 1
  for (int it0 = threadIdx.x; ks > 1 && it0 < items; it0 += 2 * kGemmThreads) {
    float4 part[2][kGemmMaxSplit], rr[2];  // both items' loads issued before the first add
    float rs[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int it = it0 + u * kGemmThreads;
      if (it < items) {
        const int j = j0 + it / (kGemmBM / 4), r4 = (it % (kGemmBM / 4)) * 4;
        const uint32_t off = red_base + 4u * (kGemmBM * j + r4);
#pragma unroll
        for (int z = 0; z < kGemmMaxSplit; ++z)
          if (z < ks) part[u][z] = ld_dsmem_f32x4(mapa_shared(off, z));
        rs[u] = g.ss_in != nullptr ? s_rs[j] : 1.f;
        if (EPI == EPI_RESID_F32 && n0 + j < g.N)
          rr[u] = __ldcg(reinterpret_cast<const float4*>(g.resid + static_cast<size_t>(n0 + j) * g.ldy + m0 + r4));
      }
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int it = it0 + u * kGemmThreads;
      if (it < items) {
        float4 y = part[u][0];
#pragma unroll
        for (int z = 1; z < kGemmMaxSplit; ++z)
          if (z < ks) {
            y.x += part[u][z].x; y.y += part[u][z].y; y.z += part[u][z].z; y.w += part[u][z].w;
          }
        const int j = j0 + it / (kGemmBM / 4), r4 = (it % (kGemmBM / 4)) * 4;
        const int n = n0 + j, rw = m0 + r4;
        const bool live = got && n < g.N && rw < g.M;
        y.x *= rs[u]; y.y *= rs[u]; y.z *= rs[u]; y.w *= rs[u];
        if (EPI == EPI_RESID_F32 && live) {
          y.x += rr[u].x; y.y += rr[u].y; y.z += rr[u].z; y.w += rr[u].w;
        }
        if (live) gemm_store4<EPI>(g, y, rw, n);
        if (EPI == EPI_RESID_F32 && g.xg_out != nullptr) gemm_fold_item(g, y, gw, rw, n, live);
      }
    }
  }
  if (ks > 1) cluster_sync_all();  // no CTA leaves while another still reads its partial
  if (threadIdx.x == 0) gemm_stamp(g, 6);
  if (warp == 0 && lane == 0) {  // timeout paths: wait (bounded) for copies never consumed
    for (int i = issued > S ? issued - S : 0; i < issued; ++i) gemm_wait(&full[i % S], (i / S) & 1u, g.err);
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) gemm_stamp(g, 7);
  if (warp == 2) tmem_dealloc(tmem, L::TMEM_COLS);
}

}  // namespace b2d

// ---- host side -------------------------------------------------------------
#include <cudaTypedefs.h>

namespace b2d {

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 2D bf16 K-major operand [rows][inner] (row pitch inner*2 bytes), tiles of
// box_rows x 64 with 128-byte swizzle.  Rows past `rows` read as zero.
inline bool make_kmajor_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint32_t box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || (inner * 2) % 16) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {inner * 2};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(kGemmBK), box_rows};
  cuuint32_t es[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tile widths (batch rows per tile), narrowest first.
constexpr int kGemmWidths[] = {16, 32, 64, 96, 128, 256};
// The next wider tile (256 stays 256).
inline int gemm_bn_next(int bn) { return bn < 64 ? 2 * bn : bn == 64 ? 96 : bn == 96 ? 128 : 256; }
// Batch rows per tile: the smallest width covering N, at most `cap`.
inline int gemm_bn_for(int n, int cap = 256) {
  int bn = 16;
  while (bn < 256 && bn < n) bn = gemm_bn_next(bn);
  return bn < cap ? bn : cap;
}

template <int BN>
inline cudaError_t gemm_set_smem_attr() {
  static bool done[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || done[dev]) return cudaSuccess;
  const int bytes = GemmSmem<BN>::BYTES;
  cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_RESID_F32>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI_SWIGLU_BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done[dev] = true;
  return e;
}

// Clusters of `ks` CTAs of the BN-wide kernel that the device runs at once
// (occupancy query, cached per device).
template <int BN>
inline int gemm_max_clusters_t(int ks) {
  static int cache[64][kGemmMaxSplit + 1] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || ks < 1 || ks > kGemmMaxSplit) return 0;
  if (cache[dev][ks] == 0) {
    if (gemm_set_smem_attr<BN>() != cudaSuccess) return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1, 1, ks);
    cfg.blockDim = dim3(kGemmThreads);
    cfg.dynamicSmemBytes = GemmSmem<BN>::BYTES;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = static_cast<unsigned>(ks);
    cfg.attrs = at;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, gemm_tc_kernel<BN, EPI_F32>, &cfg) != cudaSuccess || n < 1) n = 1;
    cache[dev][ks] = n;
  }
  return cache[dev][ks];
}

inline int gemm_max_clusters(int bn, int ks) {
  switch (bn) {
    case 16: return gemm_max_clusters_t<16>(ks);
    case 32: return gemm_max_clusters_t<32>(ks);
    case 64: return gemm_max_clusters_t<64>(ks);
    case 96: return gemm_max_clusters_t<96>(ks);
    case 128: return gemm_max_clusters_t<128>(ks);
    default: return gemm_max_clusters_t<256>(ks);
  }
}

struct GemmPlan {
  int bn, ksplit;
};

// Tile width and K split of one projection: the narrowest tile (>= the
// batch's width, <= bn_cap unless the grid would need a second wave) whose
// tiles fit in one wave, then the largest K split whose clusters all fit at
// once.
inline GemmPlan gemm_plan(int M, int N, int K, int bn_cap) {
  const int mt = M / kGemmBM;
  int bn = gemm_bn_for(N, bn_cap);
  while (bn < 256 && mt * ((N + bn - 1) / bn) > gemm_max_clusters(bn, 1)) bn = gemm_bn_next(bn);
  const int tiles = mt * ((N + bn - 1) / bn);
  int ks = 1;
  for (int k = 2; k <= kGemmMaxSplit && k <= K / kGemmBK; ++k)
    if (tiles <= gemm_max_clusters(bn, k)) ks = k;
  // 16-row tiles already split: one split deeper than one wave allows
  // (B=8 step, gate/up split 4 instead of 3: 653 -> 623 us)
  if (bn == 16 && ks > 1 && ks < kGemmMaxSplit && ks < K / kGemmBK) ++ks;
  return {bn, ks};
}

// K split so that the grid covers the SMs about once (test hook default).
inline int gemm_ksplit_for(int M, int N, int K, int sms, int bn_cap = 256) {
  const int bn = gemm_bn_for(N, bn_cap);
  const int tiles = (M / kGemmBM) * ((N + bn - 1) / bn);
  int ks = tiles > 0 ? sms / tiles : 1;
  if (ks > kGemmMaxSplit) ks = kGemmMaxSplit;
  if (ks > K / kGemmBK) ks = K / kGemmBK;
  return ks < 1 ? 1 : ks;
}

template <int BN, int EPI>
inline cudaError_t launch_gemm_t(const CUtensorMap& wm, const CUtensorMap& xm, const GemmArgs& g, cudaStream_t st,
                                 bool pdl) {
  cudaError_t e = gemm_set_smem_attr<BN>();
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(g.M / kGemmBM, (g.N + BN - 1) / BN, g.ksplit);
  cfg.blockDim = dim3(kGemmThreads);
  cfg.dynamicSmemBytes = GemmSmem<BN>::BYTES;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  unsigned na = 0;
  if (g.ksplit > 1) {
    at[na].id = cudaLaunchAttributeClusterDimension;
    at[na].val.clusterDim.x = 1;
    at[na].val.clusterDim.y = 1;
    at[na].val.clusterDim.z = static_cast<unsigned>(g.ksplit);
    ++na;
  }
  if (pdl) {
    at[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = at;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, gemm_tc_kernel<BN, EPI>, wm, xm, g);
}

// Requires M % 128 == 0, K % 64 == 0, 1 <= ksplit <= min(8, K/64); xmap's box
// rows must equal `bn` (a supported tile width).
inline cudaError_t launch_gemm(const CUtensorMap& wm, const CUtensorMap& xm, const GemmArgs& g, int epi,
                               cudaStream_t st, bool pdl, int bn) {
  if (g.M % kGemmBM || g.K % kGemmBK || g.ksplit < 1 || g.ksplit > kGemmMaxSplit || g.ksplit > g.K / kGemmBK ||
      epi < EPI_F32 || epi > EPI_SWIGLU_BF16)
    return cudaErrorInvalidValue;
#define B2D_GEMM_CASE(BNV)                                                            \
  if (bn == BNV) {                                                                    \
    if (epi == EPI_F32) return launch_gemm_t<BNV, EPI_F32>(wm, xm, g, st, pdl);       \
    if (epi == EPI_RESID_F32) return launch_gemm_t<BNV, EPI_RESID_F32>(wm, xm, g, st, pdl); \
    return launch_gemm_t<BNV, EPI_SWIGLU_BF16>(wm, xm, g, st, pdl);                   \
  }
  B2D_GEMM_CASE(16)
  B2D_GEMM_CASE(32)
  B2D_GEMM_CASE(64)
  B2D_GEMM_CASE(96)
  B2D_GEMM_CASE(128)
  B2D_GEMM_CASE(256)
#undef B2D_GEMM_CASE
  return cudaErrorInvalidValue;
}

}  // namespace b2d
