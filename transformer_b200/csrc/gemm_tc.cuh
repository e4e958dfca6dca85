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
// CTA = 4 warps: warp 0 TMA producer, warp 1 MMA issuer, warp 2 TMEM
// allocator, all four the epilogue (warp w owns TMEM lanes 32w..32w+31).
// Grid = (M/128, ceil(N/BN)).  Every wait is bounded; on expiry the kernel
// records an error word and leaves through the normal exit (TMEM freed).
#pragma once

#include <cuda_bf16.h>

#include "tc_ptx.cuh"

namespace b2d {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle atom of bf16
constexpr int kGemmStages = 6;
constexpr int kGemmThreads = 128;
constexpr uint64_t kGemmWaitNs = 200000000ull;  // 200 ms

enum : int { EPI_F32 = 0, EPI_RESID_F32 = 1, EPI_SWIGLU_BF16 = 2 };

struct GemmArgs {
  int M, N, K;
  float* y;                 // EPI_F32 / EPI_RESID_F32: [N][ldy] f32
  const float* resid;       // EPI_RESID_F32: [N][ldy] (may equal y)
  __nv_bfloat16* ybf;       // EPI_SWIGLU_BF16: [N][ldy] bf16, column m/2
  int ldy;
  uint32_t* err;            // status word: set (if still 0) when a wait runs out
};

template <int BN>
struct GemmSmem {
  static constexpr int A_BYTES = kGemmBM * kGemmBK * 2;  // 16 KB
  static constexpr int B_BYTES = BN * kGemmBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BARS = kGemmStages * STAGE;
  static constexpr int BYTES = BARS + (2 * kGemmStages + 1) * 8 + 16 + 1024;  // + alignment slack
  static constexpr uint32_t TMEM_COLS = BN < 32 ? 32 : BN;
  static_assert(STAGE % 1024 == 0, "stages must keep 1024-byte alignment for the swizzle atoms");
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

template <int BN, int EPI>
__global__ void __launch_bounds__(kGemmThreads, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
               const GemmArgs g) {
  using L = GemmSmem<BN>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::BARS);
  uint64_t* empty = full + kGemmStages;
  uint64_t* done = empty + kGemmStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kGemmBM, n0 = blockIdx.y * BN;
  const int nk = g.K / kGemmBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGemmStages; ++s) {
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

  if (warp == 0 && lane == 0) {
    // ---- TMA producer ----
    const uint64_t pol_w = l2_policy_evict_first();
    const uint64_t pol_x = l2_policy_evict_last();
    for (int kb = 0; kb < nk; ++kb) {
      const int s = kb % kGemmStages;
      if (kb >= kGemmStages && !gemm_wait(&empty[s], ((kb / kGemmStages) - 1) & 1u, g.err)) break;
      uint8_t* a = sm + s * L::STAGE;
      mbar_arrive_expect_tx(&full[s], L::STAGE);
      tma_load_2d(a, &wmap, kb * kGemmBK, m0, &full[s], pol_w);
      tma_load_2d(a + L::A_BYTES, &xmap, kb * kGemmBK, n0, &full[s], pol_x);
    }
  } else if (warp == 1 && lane == 0) {
    // ---- MMA issuer ----
    const uint32_t idesc = idesc_bf16_f32(kGemmBM, BN);
    bool ok = true;
    for (int kb = 0; kb < nk && ok; ++kb) {
      const int s = kb % kGemmStages;
      ok = gemm_wait(&full[s], (kb / kGemmStages) & 1u, g.err);
      if (!ok) break;
      tc_fence_after();
      const uint32_t a = smem_addr(sm + s * L::STAGE);
      const uint32_t b = a + L::A_BYTES;
#pragma unroll
      for (int k = 0; k < kGemmBK / 16; ++k)
        tc_mma_bf16(tmem, sdesc_kmajor_sw128(a + 32 * k), sdesc_kmajor_sw128(b + 32 * k), idesc, kb > 0 || k > 0);
      tc_commit(&empty[s]);  // stage reusable once these MMAs have read it
    }
    tc_commit(done);  // accumulator complete (or the issued part of it)
  }

  // ---- epilogue: all four warps ----
  __syncwarp();
  const bool got = __all_sync(0xffffffffu, gemm_wait(done, 0, g.err));
  tc_fence_after();
  const int row = m0 + warp * 32 + lane;  // weight row = output column m
#pragma unroll 1
  for (int c0 = 0; c0 < BN; c0 += 32) {
    float v[32];
    tmem_ld32(tmem + (static_cast<uint32_t>(warp * 32) << 16) + c0, v);
    if (!got) continue;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const int n = n0 + c0 + j;
      if (EPI == EPI_SWIGLU_BF16) {
        const float up = __shfl_xor_sync(0xffffffffu, v[j], 1);
        if (c0 + j < BN && n < g.N && (lane & 1) == 0 && row < g.M) {
          const float act = v[j] * (1.0f / (1.0f + __expf(-v[j]))) * up;
          g.ybf[static_cast<size_t>(n) * g.ldy + (row >> 1)] = __float2bfloat16_rn(act);
        }
      } else if (c0 + j < BN && n < g.N && row < g.M) {
        float out = v[j];
        if (EPI == EPI_RESID_F32) out += g.resid[static_cast<size_t>(n) * g.ldy + row];
        g.y[static_cast<size_t>(n) * g.ldy + row] = out;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
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

inline int gemm_bn_for(int n) { return n <= 16 ? 16 : (n <= 32 ? 32 : 64); }

template <int BN, int EPI>
inline cudaError_t launch_gemm_t(const CUtensorMap& wm, const CUtensorMap& xm, const GemmArgs& g, cudaStream_t st) {
  static bool attr[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(gemm_tc_kernel<BN, EPI>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         GemmSmem<BN>::BYTES);
    if (e != cudaSuccess) return e;
    attr[dev] = true;
  }
  dim3 grid(g.M / kGemmBM, (g.N + BN - 1) / BN);
  gemm_tc_kernel<BN, EPI><<<grid, kGemmThreads, GemmSmem<BN>::BYTES, st>>>(wm, xm, g);
  return cudaGetLastError();
}

// Requires M % 128 == 0 and K % 64 == 0; xmap's box rows must equal
// gemm_bn_for(N).
inline cudaError_t launch_gemm(const CUtensorMap& wm, const CUtensorMap& xm, const GemmArgs& g, int epi,
                               cudaStream_t st) {
  const int bn = gemm_bn_for(g.N);
#define B2D_GEMM_CASE(BNV)                                                       \
  if (bn == BNV) {                                                               \
    if (epi == EPI_F32) return launch_gemm_t<BNV, EPI_F32>(wm, xm, g, st);       \
    if (epi == EPI_RESID_F32) return launch_gemm_t<BNV, EPI_RESID_F32>(wm, xm, g, st); \
    return launch_gemm_t<BNV, EPI_SWIGLU_BF16>(wm, xm, g, st);                   \
  }
  B2D_GEMM_CASE(16)
  B2D_GEMM_CASE(32)
  B2D_GEMM_CASE(64)
#undef B2D_GEMM_CASE
  return cudaErrorInvalidValue;
}

}  // namespace b2d
