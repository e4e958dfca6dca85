// b2d_ptx.cuh — small inline-PTX helpers shared by the decode kernels (sm_100a).
//
// Everything here is hand-written PTX for: mbarriers, the bulk (non-tensor)
// global->shared async copy with an L2 cache-policy hint, relaxed gpu-scope
// loads/stores used by the inter-CTA exchange words, and the global timer used
// to bound every wait.  No multicast form of any copy is used.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace b2d {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ----------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// True once the phase with the given parity has completed.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// ---- bulk async copy global -> shared (completes on an mbarrier) --------
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_addr(dst)), "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy) : "memory");
}

// ---- 16-byte asynchronous copies (LSU path, not the tensor-copy unit) -------
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async16(void* dst, const void* src) { cp_async16(smem_addr(dst), src); }
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---- exchange words -----------------------------------------------------
// An exchange word is 8 bytes: low 32 bits payload (float bits), high 32 bits
// the launch's flag.  It is written with one 64-bit atomic exchange (single-copy
// atomic, so a reader that sees the current flag also sees the payload written
// with it).  The atomic is performed at L2 at once and its old value is never
// read, so the writer does not wait for it: measured on the B=1 step, a plain
// relaxed store reached the polling CTAs 2-3 us later, and a fence after the
// store made the writer itself wait ~1 us.
__device__ __forceinline__ void st_word(uint64_t* p, float v, uint32_t flag) {
  const uint64_t w = (static_cast<uint64_t>(flag) << 32) | __float_as_uint(v);
  uint64_t old;
  asm volatile("atom.relaxed.gpu.global.exch.b64 %0, [%1], %2;" : "=l"(old) : "l"(p), "l"(w) : "memory");
}
// Two adjacent words (16-byte aligned); each 64-bit element is read atomically.
__device__ __forceinline__ void ld_words2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint64_t ld_acquire_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.release.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// Orders this thread's (acquired) view of generic-proxy memory before its
// later async-proxy (bulk copy) accesses.
__device__ __forceinline__ void fence_proxy_async_all() { asm volatile("fence.proxy.async;" ::: "memory"); }
// Orders this thread's earlier generic-proxy accesses of shared memory before
// later async-proxy (bulk / tensor copy) accesses of it.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ uint32_t ld_relaxed_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t word_flag(uint64_t w) { return static_cast<uint32_t>(w >> 32); }
__device__ __forceinline__ float word_val(uint64_t w) { return __uint_as_float(static_cast<uint32_t>(w)); }

// ---- fixed-point accumulator words ----------------------------------------
// A residual-stream element that several CTAs contribute to is an 8-byte
// accumulator: bits 58..63 count the contributions, bits 0..57 hold the sum
// of (value * 2^32 + 2^51) over them.  Every contribution is one 64-bit
// atomic add, so the sum is exact and independent of the order in which the
// adds land (integer addition), and a reader that sees the expected count has
// the complete sum.  |value| < 2^19 per contribution; at most 63
// contributions (63 * 2^52 < 2^58, so the biased sum never carries into the
// count).
constexpr int kAccCountShift = 58;
constexpr uint64_t kAccBias = 1ull << 51;
constexpr float kAccLimit = 524288.f;  // 2^19
__device__ __forceinline__ void red_add_u64(uint64_t* p, uint64_t v) {
  asm volatile("red.relaxed.gpu.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
// value -> fixed point (round to nearest); false when out of range or NaN.
__device__ __forceinline__ bool acc_fix(float v, int64_t& q) {
  const bool in = fabsf(v) < kAccLimit;
  q = in ? __float2ll_rn(v * 4294967296.f) : 0;
  return in;
}
// One contribution of fixed-point q (|q| < 2^51).
__device__ __forceinline__ void acc_add(uint64_t* p, int64_t q) {
  red_add_u64(p, (1ull << kAccCountShift) + static_cast<uint64_t>(q + static_cast<int64_t>(kAccBias)));
}
__device__ __forceinline__ uint32_t acc_count(uint64_t w) { return static_cast<uint32_t>(w >> kAccCountShift); }
// The exact fixed-point sum of a word whose count is n.
__device__ __forceinline__ int64_t acc_sum(uint64_t w, uint32_t n) {
  return static_cast<int64_t>(w & ((1ull << kAccCountShift) - 1)) - static_cast<int64_t>(n) * static_cast<int64_t>(kAccBias);
}
// Nearest f32 of a fixed-point sum.
__device__ __forceinline__ float acc_value(int64_t s) { return __ll2float_rn(s) * 2.3283064365386963e-10f; }

// ---- distributed shared memory (cluster) signalling ---------------------------
// Asynchronous store into cluster CTA shared memory (addresses from mapa)
// that completes `bytes` of a transaction on the receiver's mbarrier: the
// receiver arms the phase with arrive.expect_tx(total bytes) and its wait
// completes once every pushed byte has landed.  No fence on the sender.
__device__ __forceinline__ void st_async_f32(uint32_t addr, float v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(addr), "f"(v),
               "r"(bar) : "memory");
}
__device__ __forceinline__ void st_async_f32x2(uint32_t addr, float a, float b, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
               "f"(a), "f"(b), "r"(bar) : "memory");
}
__device__ __forceinline__ void st_async_f32x4(uint32_t addr, float4 v, uint32_t bar) {
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
               "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar) : "memory");
}
// Phase test with cluster-scope acquire (the phase of a barrier that peers push to).
__device__ __forceinline__ bool mbar_test_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_addr(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// ---- named barrier among the consumer warps -----------------------------
template <int NT>
__device__ __forceinline__ void consumer_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(NT) : "memory");
}
// Barrier + AND-reduction of a predicate over the consumer threads.
template <int NT>
__device__ __forceinline__ bool consumer_sync_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r) : "r"(static_cast<uint32_t>(v)), "n"(NT) : "memory");
  return r != 0;
}

// ---- math helpers -------------------------------------------------------
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float round_bf16(float x) {
  return __bfloat162float(__float2bfloat16_rn(x));
}
// acc += dot(8 bf16 weights packed in w, 8 bf16 activations packed in x),
// products and accumulation in f32 (bf16 -> f32 is exact).
__device__ __forceinline__ float dot8(const uint4 w, const uint4 x, float acc) {
  acc = fmaf(bf16_lo(w.x), bf16_lo(x.x), acc);
  acc = fmaf(bf16_hi(w.x), bf16_hi(x.x), acc);
  acc = fmaf(bf16_lo(w.y), bf16_lo(x.y), acc);
  acc = fmaf(bf16_hi(w.y), bf16_hi(x.y), acc);
  acc = fmaf(bf16_lo(w.z), bf16_lo(x.z), acc);
  acc = fmaf(bf16_hi(w.z), bf16_hi(x.z), acc);
  acc = fmaf(bf16_lo(w.w), bf16_lo(x.w), acc);
  acc = fmaf(bf16_hi(w.w), bf16_hi(x.w), acc);
  return acc;
}
// ---- packed f32x2 arithmetic (sm_100: fma.rn.f32x2) ----------------------
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
// bf16x2 word -> (lo, hi) as f32x2 (exact)
__device__ __forceinline__ uint64_t bf2pack(uint32_t w) {
  uint64_t r;
  asm("{\n\t.reg .b32 l, h;\n\tshl.b32 l, %1, 16;\n\tand.b32 h, %1, 0xffff0000;\n\tmov.b64 %0, {l, h};\n\t}"
      : "=l"(r) : "r"(w));
  return r;
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ float f2sum(uint64_t v) {
  float lo, hi;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
  return lo + hi;
}
// 8 bf16 weights (w) times 8 f32 activations (xa: elements 0-3, xb: 4-7),
// accumulated into two f32x2 accumulators.
__device__ __forceinline__ void dot8x2(const uint4 w, const float4 xa, const float4 xb, uint64_t& a0,
                                       uint64_t& a1) {
  a0 = ffma2(bf2pack(w.x), f2pack(xa.x, xa.y), a0);
  a1 = ffma2(bf2pack(w.y), f2pack(xa.z, xa.w), a1);
  a0 = ffma2(bf2pack(w.z), f2pack(xb.x, xb.y), a0);
  a1 = ffma2(bf2pack(w.w), f2pack(xb.z, xb.w), a1);
}

// Pack two f32 (already bf16-representable) into a bf16x2 word.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  return (__float_as_uint(lo) >> 16) | (__float_as_uint(hi) & 0xffff0000u);
}

// ---- warp-level tensor-core MMA (sm_80+ forms, valid on sm_100a) ------------
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
// Programmatic dependent launch: wait for the preceding kernel's results /
// allow the next kernel's CTAs to start their prologue.  No-ops when the
// launch carries no programmatic dependency.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace b2d
