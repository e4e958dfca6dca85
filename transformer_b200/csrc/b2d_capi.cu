// b2d_capi.cu — the C ABI declared in include/b2d.h.
//
// Host side of the engine: model / workspace lifetime, layout queries, host
// validation, and the cooperative launch of the shape-specialised kernels.
// Nothing here allocates per step; workspaces are allocated once.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <new>
#include <utility>

#include "../../include/b2d.h"
#include "attn_paged.cuh"
#include "batched.cuh"
#include "decode_b1.cuh"
#include "decode_b1c.cuh"
#include "gemm_tc.cuh"
#include "sampler.cuh"

namespace {

thread_local char g_cuda_err[256] = "";

b2d_status cuda_fail(cudaError_t e, const char* what) {
  std::snprintf(g_cuda_err, sizeof(g_cuda_err), "%s: %s", what, cudaGetErrorString(e));
  if (e == cudaErrorMemoryAllocation) return B2D_ERR_NO_MEMORY;
  if (e == cudaErrorCooperativeLaunchTooLarge) return B2D_ERR_LAUNCH;
  return B2D_ERR_CUDA;
}

#define B2D_CUDA(call, what)                         \
  do {                                               \
    cudaError_t e_ = (call);                         \
    if (e_ != cudaSuccess) return cuda_fail(e_, what); \
  } while (0)

constexpr uint64_t align256(uint64_t x) { return (x + 255) & ~uint64_t(255); }

using Shape306M = b2d::Shape<1024, 2816, 16, 4>;
using ShapeTiny = b2d::Shape<256, 768, 4, 2>;

// Shape-specialised entry points.
struct ShapeOps {
  int d, dff, nh, nkv;
  int (*chunk_begin)(int c, int G);  // the cluster kernel's act-chunk split
  size_t smem;
  const void* kernel;        // the B=1 step, flat grid (one CTA per SM)
  const void* kernel_trace;  // the same with diagnostic stamps (b2d_debug_trace, knobs 7/8)
  size_t smem_c;
  const void* kernel_c;        // the B=1 step on clusters of kCS CTAs (decode_b1c.cuh)
  const void* kernel_c_trace;
  int qbox, obox, gbox, dbox;  // the cluster kernel's q/k/v, Wo, gate/up, Wd tensor-copy rows
};

template <class S>
int chunk_begin_host(int c, int G) { return b2d::chunk_begin<S>(c, G); }

template <class S>
ShapeOps make_ops() {
  return ShapeOps{S::D, S::DFF, S::NH, S::NKV, &chunk_begin_host<S>, sizeof(b2d::Smem<S>),
                  reinterpret_cast<const void*>(&b2d::decode_b1_kernel<S, false>),
                  reinterpret_cast<const void*>(&b2d::decode_b1_kernel<S, true>),
                  b2d::smem_c_bytes<S>(),
                  reinterpret_cast<const void*>(&b2d::decode_b1c_kernel<S, false>),
                  reinterpret_cast<const void*>(&b2d::decode_b1c_kernel<S, true>),
                  b2d::ShapeC<S>::QPS, b2d::ShapeC<S>::OBOX, b2d::ShapeC<S>::PS, b2d::ShapeC<S>::DBOX};
}

// Tensor map of one projection over all layers: [n_layers][rows][inner] bf16
// (row pitch inner * 2 bytes, layer pitch layer_stride), boxes of box_inner x
// box_rows x 1.
bool make_layer_map(CUtensorMap* map, const void* base, uint64_t inner, uint64_t rows, uint64_t layers,
                    uint64_t layer_stride, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  auto enc = b2d::tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || (inner * 2) % 16 || layer_stride % 16) return false;
  cuuint64_t dims[3] = {inner, rows, layers};
  cuuint64_t strides[2] = {inner * 2, layer_stride};
  cuuint32_t box[3] = {box_inner, box_rows, 1};
  cuuint32_t es[3] = {1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Row-major projection [n_layers][rows][k] bf16 viewed as k-blocks: {64, rows,
// k / 64, n_layers} with strides {k * 2, 128, layer_stride}; a box of
// box_rows rows lands as [k / 64][box_rows][64], 128-byte swizzled.
bool make_kblock_map(CUtensorMap* map, const void* base, uint64_t k, uint64_t rows, uint64_t layers,
                     uint64_t layer_stride, uint32_t box_rows) {
  auto enc = b2d::tensor_map_encoder();
  if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || k % 64 || layer_stride % 16 || k / 64 > 256) return false;
  cuuint64_t dims[4] = {64, rows, k / 64, layers};
  cuuint64_t strides[3] = {k * 2, 128, layer_stride};
  cuuint32_t box[4] = {64, box_rows, static_cast<cuuint32_t>(k / 64), 1};
  cuuint32_t es[4] = {1, 1, 1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, es,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The cluster kernel's weight views of the packed weights as stored: q/k/v
// and gate/up rows in k-block boxes, Wo boxes of 64 columns (one head) x obox
// rows (128-byte swizzled), Wd boxes of 8 columns (one act chunk) x dbox rows.
bool make_b1c_maps(const b2d_config* c, const ShapeOps* ops, const uint8_t* w, const b2d_weights_layout_t& lay,
                   b2d::MapsC* maps) {
  const uint64_t d = c->d_model, f = c->d_ff, nl = c->n_layers;
  const uint64_t qkv = uint64_t(c->n_heads + 2 * c->n_kv_heads) * c->d_head;
  return make_kblock_map(&maps->qkv, w + lay.off_qkv, d, qkv, nl, lay.layer_stride, uint32_t(ops->qbox)) &&
         make_layer_map(&maps->o, w + lay.off_o, d, d, nl, lay.layer_stride, 64, uint32_t(ops->obox),
                        CU_TENSOR_MAP_SWIZZLE_128B) &&
         make_kblock_map(&maps->gu, w + lay.off_gu, d, 2 * f, nl, lay.layer_stride, uint32_t(ops->gbox)) &&
         make_layer_map(&maps->down, w + lay.off_down, f, d, nl, lay.layer_stride, 8, uint32_t(ops->dbox),
                        CU_TENSOR_MAP_SWIZZLE_NONE);
}

// Clusters of the cluster kernel that fit co-resident (0 if none / unsupported).
int b1c_max_clusters(const ShapeOps* ops) {
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = b2d::kCS;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  cfg.gridDim = dim3(b2d::kCS * 64);
  cfg.blockDim = dim3(b2d::kThreads);
  cfg.dynamicSmemBytes = ops->smem_c;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, ops->kernel_c, &cfg) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

// Grid of the cluster kernel for this shape on the current device, or 0 when
// it does not fit (the flat kernel is used then).
int b1c_grid(const ShapeOps* ops) {
  const int nc = b1c_max_clusters(ops);
  if (nc < ops->nh || nc * b2d::kCS < b2d::kMinGridC) return 0;
  const int grid = nc * b2d::kCS;
  for (int c = 0; c < grid; ++c)  // the kernel's per-CTA gate/up budget
    if (ops->chunk_begin(c + 1, grid) - ops->chunk_begin(c, grid) > b2d::kMaxChunksC) return 0;
  return grid;
}

// One cooperative launch of the cluster kernel.
cudaError_t launch_b1c(const void* kernel, int grid, size_t smem, cudaStream_t st, const b2d::MapsC& maps,
                       const b2d::DecodeArgs& A, bool cooperative = true) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(b2d::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = b2d::kCS;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeCooperative;
  at[1].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = cooperative ? 2 : 1;
  void* args[] = {const_cast<b2d::MapsC*>(&maps), const_cast<b2d::DecodeArgs*>(&A)};
  return cudaLaunchKernelExC(&cfg, kernel, args);
}

const ShapeOps* find_ops(const b2d_config* c) {
  static const ShapeOps ops[] = {make_ops<Shape306M>(), make_ops<ShapeTiny>()};
  if (!c || c->d_head != 64) return nullptr;
  for (const auto& o : ops)
    if (o.d == c->d_model && o.dff == c->d_ff && o.nh == c->n_heads && o.nkv == c->n_kv_heads) return &o;
  return nullptr;
}

bool config_valid(const b2d_config* c) {
  return c && c->vocab_size > 0 && c->d_model > 0 && c->n_heads > 0 && c->n_kv_heads > 0 &&
         c->n_layers > 0 && c->d_head == 64 && c->d_ff > 0 && c->context_len > 0 &&
         c->n_heads % c->n_kv_heads == 0 && c->rms_eps > 0.f;
}

void compute_layout(const b2d_config* c, b2d_weights_layout_t* L) {
  const uint64_t d = c->d_model, f = c->d_ff, qkv = uint64_t(c->n_heads + 2 * c->n_kv_heads) * c->d_head;
  const uint64_t V = c->vocab_size, nl = c->n_layers, half = c->d_head / 2, ctx = c->context_len;
  L->off_qkv = 0;
  L->off_o = L->off_qkv + align256(qkv * d * 2);
  L->off_gu = L->off_o + align256(d * d * 2);
  L->off_down = L->off_gu + align256(f * 2 * d * 2);
  L->layer_stride = L->off_down + align256(d * f * 2);
  L->off_emb = nl * L->layer_stride;
  L->off_ln1 = L->off_emb + align256(V * d * 2);
  L->off_ln2 = L->off_ln1 + align256(nl * d * 4);
  L->off_lnf = L->off_ln2 + align256(nl * d * 4);
  L->off_cos = L->off_lnf + align256(d * 4);
  L->off_sin = L->off_cos + align256(ctx * half * 4);
  L->total_bytes = L->off_sin + align256(ctx * half * 4);
}

}  // namespace

struct b2d_model {
  b2d_config cfg;
  int device;
  const uint8_t* w;
  uint64_t wbytes;
  b2d_weights_layout_t lay;
  const ShapeOps* ops;
  int grid;               // SMs (the flat B=1 kernel's grid)
  int b1_grid;            // the cluster B=1 kernel's grid (0 = the flat kernel is used)
  b2d::MapsC b1_maps;     // its weight views
  // batched path: TMA descriptors of every projection (created on first use)
  bool maps_ready;
  CUtensorMap* wmaps;  // [4 * n_layers + 1]: per layer qkv, o, gu, down; then the embedding
};

struct b2d_ws {
  b2d_model* m;
  int max_batch;
  uint64_t* words;
  size_t n_words;
  b2d::Control* ctl;
  float* am_val;
  int32_t* am_idx;
  uint32_t layer_words, w_att, w_hm, w_act;
  int att_T;
  uint64_t wait_ns;
  int extra_ctas;          // test hook: work split over this many CTAs more than launched
  bool force_flat;         // diagnostics: B=1 step on the flat kernel even where clusters fit
  uint64_t* acc;           // cluster kernel: residual accumulators [2][2 n_layers][d_model]
  size_t acc_words;
  int b1_kind;             // kernel of the last B=1 launch: 0 none / flat, 1 cluster
  uint64_t* trace;
  int trace_stride;
  uint32_t poll_ns;
  int max_inflight;
  // batched path and prefill: buffers for brows = max(max_batch, kPrefillRows) rows
  int brows;
  int32_t* prefill_pos;            // [kPrefillRows] positions of a prefill chunk
  int last_launches;               // kernels launched by the last batched step / prefill chunk
  int rows;                        // activation rows allocated (max_batch rounded up to the widest tile)
  float *H, *Hm, *qkv, *logits;
  float* ss;               // folded RMSNorm: per-tile sums of squares [d_model / 128][rows]
  bool no_pdl;             // diagnostics: launch without programmatic dependencies
  int force_ksplit;        // diagnostics: fixed K split (0 = automatic)
  int force_att_cpc;       // diagnostics: fixed attention units per (sequence, kv head) (0 = automatic)
  uint64_t* gemm_trace;    // diagnostics: [launch][kTraceCtas][kGemmStamps] projection stamps, or null
  uint64_t* stage_trace;   // diagnostics: B=1 stage stamps [grid][3][stage_stride], or null
  uint64_t* att_trace;     // diagnostics: attention stamps [layer][kAttTraceUnits][8], or null
  uint64_t* sample_trace;  // diagnostics: sampler phase stamps [batch][8], or null
  uint64_t* sample_scratch;  // top-p sort buffer [sample_rows][kSamplerMaxVocab]
  int sample_rows;
  int sample_mode;         // diagnostics: top-p kernel choice (0 automatic, 1 one CTA, 2 clusters of 8)
  bool b1_plain;           // diagnostics: the B=1 cluster grid launched without the cooperative attribute
  int32_t* tok_host;       // b2d_decode_token: mapped pinned word the kernel writes the argmax to
  int32_t* tok_dev;        // its device address
  int stage_stride;
  __nv_bfloat16 *X, *A, *ACT;
  CUtensorMap xmap[6], amap[6], actmap[6];  // box rows 16 / 32 / 64 / 96 / 128 / 256 (bn_index)
  // b2d_decode_step_paged: CUDA graphs of the step's kernel sequence, one per
  // argument set (LRU), captured on cap_stream and launched on the caller's.
  struct StepGraph {
    const void* ptr[6];    // tok, pos, pool, table, logits, next_tok
    int batch, bps, nblk;
    uint32_t tune;         // tune_gen at capture
    int uses;              // calls seen with these arguments
    int launches;          // kernels in the graph
    uint64_t tick;         // last use
    cudaGraphExec_t exec;
  } graphs[16];
  uint64_t graph_tick;
  uint32_t tune_gen;       // bumped by every b2d_debug_tune call (cached graphs bake the knobs in)
  bool no_graph;           // step through direct launches only
  cudaStream_t cap_stream; // capture stream (created on first capture)
  // paged attention: TMA view of the last paged pool used (rows of 64 bf16)
  CUtensorMap kvmap;
  const void* kvmap_pool;
  int kvmap_nblk;
};

namespace {
constexpr int kTraceCtas = 256;        // projection CTAs stamped per launch (diagnostics)
constexpr int kTraceLaunches = 4 * 64 + 1;  // stamped projection launches per step (n_layers <= 64)
constexpr int kAttTraceUnits = 8192;        // attention units stamped per launch (diagnostics)
constexpr int kPrefillRows = 512;           // prompt positions per prefill chunk

__global__ void iota_kernel(int32_t* out, int start, int n) {
  b2d::pdl_wait();
  b2d::pdl_launch();
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = start + i;
}
inline int bn_index(int bn) { return bn == 16 ? 0 : bn == 32 ? 1 : bn == 64 ? 2 : bn == 96 ? 3 : bn == 128 ? 4 : 5; }

// Launch with an optional programmatic dependency on the previous kernel of
// the stream (the kernels call griddepcontrol.wait before reading its output).
template <typename... KArgs, typename... Args>
cudaError_t launch_k(void (*k)(KArgs...), dim3 grid, dim3 block, cudaStream_t st, bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}
// The attention kernels' dynamic shared-memory limits, raised once per device.
cudaError_t attn_smem_attrs() {
  static bool raised[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (raised[dev]) return cudaSuccess;
  cudaError_t e = cudaSuccess;
  const std::pair<const void*, int> ks[] = {
      {reinterpret_cast<const void*>(&b2d::paged_attn_mma_kernel<2, false>), b2d::pa_smem_bytes(2, false)},
      {reinterpret_cast<const void*>(&b2d::paged_attn_mma_kernel<4, false>), b2d::pa_smem_bytes(4, false)},
      {reinterpret_cast<const void*>(&b2d::paged_attn_mma_kernel<2, true>), b2d::pa_smem_bytes(2, true)},
      {reinterpret_cast<const void*>(&b2d::paged_attn_mma_kernel<4, true>), b2d::pa_smem_bytes(4, true)},
      {reinterpret_cast<const void*>(&b2d::paged_attn_mma_kernel<2, true, b2d::kPaStagesShallow>),
       b2d::pa_smem_bytes(2, true, b2d::kPaStagesShallow)},
      {reinterpret_cast<const void*>(&b2d::paged_attn_mma_kernel<2, true, b2d::kPaStagesSplit>),
       b2d::pa_smem_bytes(2, true, b2d::kPaStagesSplit)}};
  for (const auto& k : ks)
    if (e == cudaSuccess) e = cudaFuncSetAttribute(k.first, cudaFuncAttributeMaxDynamicSharedMemorySize, k.second);
  if (e == cudaSuccess) raised[dev] = true;
  return e;
}

// launch_k with `smem` bytes of dynamic shared memory (the caller has raised
// the kernel's limit where it exceeds the default).
template <class... KArgs, class... Args>
cudaError_t launch_k_smem(void (*k)(KArgs...), dim3 grid, dim3 block, int smem, cudaStream_t st, bool pdl,
                          Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k, std::forward<Args>(args)...);
}
}  // namespace

extern "C" {

const char* b2d_status_str(b2d_status s) {
  switch (s) {
    case B2D_OK: return "ok";
    case B2D_ERR_INVALID_ARG: return "invalid argument";
    case B2D_ERR_UNSUPPORTED: return "model shape or batch not supported by this build";
    case B2D_ERR_CUDA: return "CUDA error";
    case B2D_ERR_NO_MEMORY: return "out of device memory";
    case B2D_ERR_LAUNCH: return "cooperative launch refused (grid not co-resident)";
    case B2D_ERR_DEVICE_TIMEOUT: return "device wait timed out";
    case B2D_ERR_DEVICE_INPUT: return "device saw token/pos out of range";
    case B2D_ERR_DEVICE_HALTED: return "workspace halted by an earlier device error";
    case B2D_ERR_SCRATCH_LIMIT: return "model needs more scratch than the no-allocation entry point's fixed 4 MiB array";
  }
  return "unknown status";
}

const char* b2d_cuda_error(void) { return g_cuda_err; }

int b2d_config_supported(const b2d_config* cfg) { return config_valid(cfg) && find_ops(cfg) ? 1 : 0; }

b2d_status b2d_weights_layout(const b2d_config* cfg, b2d_weights_layout_t* out) {
  if (!config_valid(cfg) || !out) return B2D_ERR_INVALID_ARG;
  compute_layout(cfg, out);
  return B2D_OK;
}

b2d_status b2d_kv_layout(const b2d_config* cfg, b2d_kv_layout_t* out) {
  if (!config_valid(cfg) || !out) return B2D_ERR_INVALID_ARG;
  out->kv_half_elems = uint64_t(cfg->n_kv_heads) * cfg->context_len * cfg->d_head;
  out->layer_elems = 2 * out->kv_half_elems;
  out->elems_per_seq = uint64_t(cfg->n_layers) * out->layer_elems;
  return B2D_OK;
}

b2d_status b2d_model_create(const b2d_config* cfg, const void* weights_dev, uint64_t weights_bytes,
                            int device, b2d_model** out) {
  if (!out) return B2D_ERR_INVALID_ARG;
  *out = nullptr;
  if (!config_valid(cfg) || !weights_dev || (reinterpret_cast<uintptr_t>(weights_dev) & 255u))
    return B2D_ERR_INVALID_ARG;
  const ShapeOps* ops = find_ops(cfg);
  if (!ops) return B2D_ERR_UNSUPPORTED;
  b2d_weights_layout_t lay;
  compute_layout(cfg, &lay);
  if (weights_bytes < lay.total_bytes) return B2D_ERR_INVALID_ARG;
  int ndev = 0;
  B2D_CUDA(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
  if (device < 0 || device >= ndev) return B2D_ERR_INVALID_ARG;
  B2D_CUDA(cudaSetDevice(device), "cudaSetDevice");
  int sms = 0, coop = 0;
  B2D_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "sm count");
  B2D_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device), "coop attr");
  if (!coop) return B2D_ERR_LAUNCH;
  for (const void* k : {ops->kernel, ops->kernel_trace})
    B2D_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(ops->smem)),
             "cudaFuncSetAttribute(smem)");
  for (const void* k : {ops->kernel_c, ops->kernel_c_trace})
    B2D_CUDA(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(ops->smem_c)),
             "cudaFuncSetAttribute(smem)");
  if (sms < b2d::kMinGrid) return B2D_ERR_UNSUPPORTED;  // phase register budgets assume >= 128 SMs
  int per_sm = 0;
  B2D_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ops->kernel, b2d::kThreads, ops->smem),
           "occupancy");
  if (per_sm < 1) return B2D_ERR_LAUNCH;
  b2d_model* m = new (std::nothrow) b2d_model;
  if (!m) return B2D_ERR_NO_MEMORY;
  m->cfg = *cfg;
  m->device = device;
  m->w = static_cast<const uint8_t*>(weights_dev);
  m->wbytes = weights_bytes;
  m->lay = lay;
  m->ops = ops;
  m->grid = sms;
  m->b1_grid = b1c_grid(ops);
  if (m->b1_grid > 0 && !make_b1c_maps(cfg, ops, m->w, lay, &m->b1_maps)) m->b1_grid = 0;
  m->maps_ready = false;
  m->wmaps = nullptr;
  *out = m;
  return B2D_OK;
}

b2d_status b2d_model_destroy(b2d_model* m) {
  if (m) delete[] m->wmaps;
  delete m;
  return B2D_OK;
}

int b2d_model_grid(const b2d_model* m) { return m ? (m->b1_grid > 0 ? m->b1_grid : m->grid) : 0; }

b2d_status b2d_workspace_create(b2d_model* m, int max_batch, b2d_ws** out) {
  if (!out) return B2D_ERR_INVALID_ARG;
  *out = nullptr;
  if (!m || max_batch < 1) return B2D_ERR_INVALID_ARG;
  B2D_CUDA(cudaSetDevice(m->device), "cudaSetDevice");
  const b2d_config& c = m->cfg;
  b2d_ws* ws = new (std::nothrow) b2d_ws;
  if (!ws) return B2D_ERR_NO_MEMORY;
  std::memset(ws, 0, sizeof(*ws));
  ws->m = m;
  ws->max_batch = max_batch;
  ws->att_T = 128 * ((c.context_len + 511) / 512);  // <= kMaxSplits units per head
  const uint32_t qkv = uint32_t(c.n_heads + 2 * c.n_kv_heads) * 64;
  ws->w_att = uint32_t(c.d_model) + qkv;
  ws->w_hm = ws->w_att + uint32_t(c.n_heads) * b2d::kMaxSplits * b2d::kAttWords;
  ws->w_act = ws->w_hm + uint32_t(c.d_model);
  ws->layer_words = ws->w_act + uint32_t(c.d_ff);
  ws->layer_words = (ws->layer_words + 1) & ~1u;
  ws->n_words = size_t(c.n_layers) * ws->layer_words + c.d_model;
  ws->wait_ns = 2000000000ull;  // 2 s bound on every in-kernel wait
  ws->max_inflight = 4;
  ws->acc_words = size_t(2) * 2 * c.n_layers * c.d_model * b2d::kAccStride;
  cudaError_t e = cudaMalloc(&ws->words, ws->n_words * sizeof(uint64_t));
  if (e == cudaSuccess) e = cudaMalloc(&ws->acc, ws->acc_words * sizeof(uint64_t));
  if (e == cudaSuccess) e = cudaMemset(ws->acc, 0, ws->acc_words * sizeof(uint64_t));
  if (e == cudaSuccess) e = cudaMalloc(&ws->ctl, sizeof(b2d::Control));
  if (e == cudaSuccess) e = cudaMalloc(&ws->am_val, sizeof(float) * m->grid);
  if (e == cudaSuccess) e = cudaMalloc(&ws->am_idx, sizeof(int32_t) * m->grid);
  if (e == cudaSuccess) {  // batched step and prefill buffers
    ws->brows = std::max(max_batch, kPrefillRows);
    const size_t D = c.d_model, F = c.d_ff, Q = qkv, V = c.vocab_size;
    ws->rows = (ws->brows + 255) / 256 * 256;  // any tile width may be chosen (see gemm_plan)
    e = cudaMalloc(&ws->prefill_pos, sizeof(int32_t) * kPrefillRows);
    if (e == cudaSuccess) e = cudaMalloc(&ws->H, sizeof(float) * D * ws->brows);
    if (e == cudaSuccess) e = cudaMalloc(&ws->Hm, sizeof(float) * D * ws->brows);
    if (e == cudaSuccess) e = cudaMalloc(&ws->qkv, sizeof(float) * Q * ws->brows);
    if (e == cudaSuccess) e = cudaMalloc(&ws->logits, sizeof(float) * V * ws->brows);
    if (e == cudaSuccess) e = cudaMalloc(&ws->X, 2 * D * ws->rows);
    if (e == cudaSuccess) e = cudaMalloc(&ws->A, 2 * D * ws->rows);
    if (e == cudaSuccess) e = cudaMalloc(&ws->ACT, 2 * F * ws->rows);
    if (e == cudaSuccess) e = cudaMemset(ws->X, 0, 2 * D * ws->rows);
    if (e == cudaSuccess) e = cudaMemset(ws->A, 0, 2 * D * ws->rows);
    if (e == cudaSuccess) e = cudaMemset(ws->ACT, 0, 2 * F * ws->rows);
    if (e == cudaSuccess) e = cudaMalloc(&ws->ss, sizeof(float) * (D / b2d::kGemmBM) * ws->rows);
    for (int i = 0; i < 6 && e == cudaSuccess; ++i) {
      const uint32_t box = static_cast<uint32_t>(b2d::kGemmWidths[i]);
      if (!b2d::make_kmajor_map(&ws->xmap[i], ws->X, D, ws->rows, box) ||
          !b2d::make_kmajor_map(&ws->amap[i], ws->A, D, ws->rows, box) ||
          !b2d::make_kmajor_map(&ws->actmap[i], ws->ACT, F, ws->rows, box))
        e = cudaErrorInvalidValue;
    }
  }
  if (e == cudaSuccess) e = cudaMemset(ws->words, 0, ws->n_words * sizeof(uint64_t));
  if (e == cudaSuccess) e = cudaMemset(ws->ctl, 0, sizeof(b2d::Control));
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    b2d_workspace_destroy(ws);
    return cuda_fail(e, "workspace allocation");
  }
  *out = ws;
  return B2D_OK;
}

b2d_status b2d_workspace_destroy(b2d_ws* ws) {
  if (!ws) return B2D_OK;
  if (ws->m) cudaSetDevice(ws->m->device);
  for (auto& g : ws->graphs)
    if (g.exec) cudaGraphExecDestroy(g.exec);
  cudaFree(ws->sample_scratch);
  cudaFreeHost(ws->tok_host);  // (tok_dev is its device alias)
  if (ws->cap_stream) cudaStreamDestroy(ws->cap_stream);
  cudaFree(ws->H);
  cudaFree(ws->Hm);
  cudaFree(ws->qkv);
  cudaFree(ws->logits);
  cudaFree(ws->X);
  cudaFree(ws->A);
  cudaFree(ws->ACT);
  cudaFree(ws->ss);
  cudaFree(ws->prefill_pos);
  cudaFree(ws->words);
  cudaFree(ws->acc);
  cudaFree(ws->ctl);
  cudaFree(ws->am_val);
  cudaFree(ws->am_idx);
  delete ws;
  return B2D_OK;
}

b2d_status b2d_workspace_reset(b2d_ws* ws, void* stream) {
  if (!ws) return B2D_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2D_CUDA(cudaSetDevice(ws->m->device), "cudaSetDevice");
  B2D_CUDA(cudaMemsetAsync(ws->words, 0, ws->n_words * sizeof(uint64_t), st), "reset words");
  B2D_CUDA(cudaMemsetAsync(ws->acc, 0, ws->acc_words * sizeof(uint64_t), st), "reset accumulators");
  B2D_CUDA(cudaMemsetAsync(ws->ctl, 0, sizeof(b2d::Control), st), "reset control");
  return B2D_OK;
}

b2d_status b2d_last_error(b2d_ws* ws, void* stream, uint32_t* detail) {
  if (!ws) return B2D_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2D_CUDA(cudaSetDevice(ws->m->device), "cudaSetDevice");
  uint32_t s = 0;
  B2D_CUDA(cudaMemcpyAsync(&s, &ws->ctl->status, sizeof(s), cudaMemcpyDeviceToHost, st), "read status");
  B2D_CUDA(cudaStreamSynchronize(st), "cudaStreamSynchronize");
  if (detail) *detail = s;
  if (s == 0) return B2D_OK;
  if ((s & 0xF00u) == b2d::ST_TIMEOUT) return B2D_ERR_DEVICE_TIMEOUT;
  if ((s & 0xF00u) == b2d::ST_BAD_INPUT) return B2D_ERR_DEVICE_INPUT;
  return B2D_ERR_DEVICE_HALTED;
}

// Test hook (not part of the product surface): shorten the in-kernel wait
// bound and/or split the work over more CTAs than are launched, so a test can
// make a wait run out on a flag nothing sets and check the status word.
b2d_status b2d_debug_set(b2d_ws* ws, uint64_t wait_ns, int extra_ctas) {
  if (!ws || wait_ns == 0 || extra_ctas < 0 || extra_ctas > 1024) return B2D_ERR_INVALID_ARG;
  ws->wait_ns = wait_ns;
  ws->extra_ctas = extra_ctas;
  return B2D_OK;
}

// Diagnostic hooks: per-CTA phase stamps (global timer, ns) into a caller
// buffer of grid * stamps_per_cta uint64 (NULL disables), and a back-off
// between failed polls of the exchange words.
b2d_status b2d_debug_trace(b2d_ws* ws, uint64_t* buf_dev, int stamps_per_cta) {
  if (!ws || stamps_per_cta < 0 || (buf_dev == nullptr) != (stamps_per_cta == 0)) return B2D_ERR_INVALID_ARG;
  ws->trace = buf_dev;
  ws->trace_stride = stamps_per_cta;
  return B2D_OK;
}

b2d_status b2d_debug_tune(b2d_ws* ws, int knob, int64_t value) {
  if (!ws) return B2D_ERR_INVALID_ARG;
  ++ws->tune_gen;  // cached step graphs hold the previous settings
  switch (knob) {
    case 12:  // B=1 step: the flat kernel (1) or the cluster kernel where it fits (0, default)
      if (value < 0 || value > 1) return B2D_ERR_INVALID_ARG;
      ws->force_flat = value == 1;
      return B2D_OK;
    case 11:  // batched step: replay cached CUDA graphs (1, default) or launch directly (0)
      if (value < 0 || value > 1) return B2D_ERR_INVALID_ARG;
      ws->no_graph = value == 0;
      return B2D_OK;
    case 1:  // back-off between failed polls, ns
      if (value < 0 || value > 100000) return B2D_ERR_INVALID_ARG;
      ws->poll_ns = static_cast<uint32_t>(value);
      return B2D_OK;
    case 2:  // bulk copies in flight per CTA
      if (value < 1 || value > b2d::kStagesC) return B2D_ERR_INVALID_ARG;  // the larger ring
      ws->max_inflight = static_cast<int>(value);
      return B2D_OK;
    case 3:  // batched step: programmatic dependent launch on (1) / off (0)
      if (value < 0 || value > 1) return B2D_ERR_INVALID_ARG;
      ws->no_pdl = value == 0;
      return B2D_OK;
    case 4:  // batched step: force the projections' K split (0 = automatic)
      if (value < 0 || value > b2d::kGemmMaxSplit) return B2D_ERR_INVALID_ARG;
      ws->force_ksplit = static_cast<int>(value);
      return B2D_OK;
    case 5:  // batched step: force the attention units per (sequence, kv head) (0 = automatic)
      if (value < 0 || value > 32) return B2D_ERR_INVALID_ARG;
      ws->force_att_cpc = static_cast<int>(value);
      return B2D_OK;
    case 6:  // batched step: projection stamp buffer (device address; 0 = off)
      ws->gemm_trace = reinterpret_cast<uint64_t*>(static_cast<uintptr_t>(value));
      return B2D_OK;
    case 7:  // B=1 step: stage stamp buffer (device address; 0 = off)
      ws->stage_trace = reinterpret_cast<uint64_t*>(static_cast<uintptr_t>(value));
      return B2D_OK;
    case 8:  // B=1 step: stage stamps per CTA and kind
      if (value < 0 || value > 4096) return B2D_ERR_INVALID_ARG;
      ws->stage_stride = static_cast<int>(value);
      return B2D_OK;
    case 9:  // batched step: attention stamp buffer (device address; 0 = off)
      ws->att_trace = reinterpret_cast<uint64_t*>(static_cast<uintptr_t>(value));
      return B2D_OK;
    case 10:  // sampler: phase stamp buffer (device address; 0 = off)
      ws->sample_trace = reinterpret_cast<uint64_t*>(static_cast<uintptr_t>(value));
      return B2D_OK;
    case 14:  // B=1 cluster kernel: plain cluster launch (1) or cooperative (0, default).  The grid is the
              // co-resident cluster count either way; profilers cannot replay a cooperative launch
      if (value < 0 || value > 1) return B2D_ERR_INVALID_ARG;
      ws->b1_plain = value == 1;
      return B2D_OK;
    case 13:  // sampler: top-p draws automatic (0, default: clusters of 16, else 8, where they fit),
              // on one CTA per sequence (1) or on clusters of 8 where they fit (2)
      if (value < 0 || value > 2) return B2D_ERR_INVALID_ARG;
      ws->sample_mode = static_cast<int>(value);
      return B2D_OK;

  }
  return B2D_ERR_INVALID_ARG;
}

namespace {
// One cooperative launch of the B=1 kernel: n_steps greedy tokens.
// tok_dev / pos_dev null: the launch carries tok_val / pos_val instead.
b2d_status launch_b1(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, const int32_t* pos_dev, void* kv_dev,
                     float* logits_dev, int32_t* next_tok_dev, int n_steps, int32_t* tok_out_dev,
                     cudaStream_t st, int32_t tok_val = 0, int32_t pos_val = 0) {
  const b2d_config& c = m->cfg;
  b2d::DecodeArgs A;
  std::memset(&A, 0, sizeof(A));
  A.wbase = m->w;
  A.layer_stride = m->lay.layer_stride;
  A.off_qkv = m->lay.off_qkv;
  A.off_o = m->lay.off_o;
  A.off_gu = m->lay.off_gu;
  A.off_down = m->lay.off_down;
  A.off_emb = m->lay.off_emb;
  A.ln1 = reinterpret_cast<const float*>(m->w + m->lay.off_ln1);
  A.ln2 = reinterpret_cast<const float*>(m->w + m->lay.off_ln2);
  A.lnf = reinterpret_cast<const float*>(m->w + m->lay.off_lnf);
  A.rcos = reinterpret_cast<const float*>(m->w + m->lay.off_cos);
  A.rsin = reinterpret_cast<const float*>(m->w + m->lay.off_sin);
  A.tok = tok_dev;
  A.pos = pos_dev;
  A.tok_val = tok_val;
  A.pos_val = pos_val;
  A.kv = static_cast<__nv_bfloat16*>(kv_dev);
  A.logits = logits_dev;
  A.next_tok = next_tok_dev;
  A.words = ws->words;
  A.acc = ws->acc;
  A.ctl = ws->ctl;
  A.am_val = ws->am_val;
  A.am_idx = ws->am_idx;
  A.layer_words = ws->layer_words;
  A.w_att = ws->w_att;
  A.w_hm = ws->w_hm;
  A.w_act = ws->w_act;
  A.vocab = c.vocab_size;
  A.n_layers = c.n_layers;
  A.ctx = c.context_len;
  A.att_T = ws->att_T;
  const bool clustered = m->b1_grid > 0 && !ws->force_flat;
  const int grid = clustered ? m->b1_grid : m->grid;
  A.grid_part = grid + ws->extra_ctas;
  A.wait_ns = ws->wait_ns;
  A.eps = c.rms_eps;
  A.trace = ws->trace;
  A.trace_stride = ws->trace_stride;
  A.stage_trace = ws->stage_trace;
  A.stage_stride = ws->stage_stride;
  A.poll_ns = ws->poll_ns;
  A.max_inflight = ws->max_inflight;
  A.n_steps = n_steps;
  A.tok_out = tok_out_dev;
  const bool trace = A.trace || A.stage_trace;
  if (clustered && ws->b1_kind != 1) {
    // The cluster kernel finds the next step's accumulators zeroed by the
    // step before it; after flat-kernel steps that is not so.
    B2D_CUDA(cudaMemsetAsync(ws->acc, 0, ws->acc_words * sizeof(uint64_t), st), "clear accumulators");
  }
  ws->b1_kind = clustered ? 1 : 0;
  if (clustered) {
    B2D_CUDA(launch_b1c(trace ? m->ops->kernel_c_trace : m->ops->kernel_c, grid, m->ops->smem_c, st, m->b1_maps, A,
                        !ws->b1_plain),
             "decode launch");
    return B2D_OK;
  }
  void* args[] = {&A};
  const void* kernel = trace ? m->ops->kernel_trace : m->ops->kernel;
  B2D_CUDA(cudaLaunchCooperativeKernel(kernel, dim3(grid), dim3(b2d::kThreads), args, m->ops->smem, st),
           "decode launch");
  return B2D_OK;
}
}  // namespace

b2d_status b2d_decode_step(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, const int32_t* pos_dev,
                           int batch, void* kv_dev, float* logits_dev, int32_t* next_tok_dev,
                           void* stream) {
  if (!m || !ws || ws->m != m || !tok_dev || !pos_dev || !kv_dev || !next_tok_dev || batch < 1 ||
      batch > ws->max_batch)
    return B2D_ERR_INVALID_ARG;
  if (batch != 1) return B2D_ERR_UNSUPPORTED;
  B2D_CUDA(cudaSetDevice(m->device), "cudaSetDevice");
  return launch_b1(m, ws, tok_dev, pos_dev, kv_dev, logits_dev, next_tok_dev, 1, nullptr,
                   static_cast<cudaStream_t>(stream));
}

b2d_status b2d_decode_token(b2d_model* m, b2d_ws* ws, int32_t tok, int32_t pos, void* kv_dev, float* logits_dev,
                            int32_t* next_tok, void* stream) {
  if (!m || !ws || ws->m != m || !kv_dev || !next_tok || tok < 0 || tok >= m->cfg.vocab_size || pos < 0 ||
      pos >= m->cfg.context_len)
    return B2D_ERR_INVALID_ARG;
  B2D_CUDA(cudaSetDevice(m->device), "cudaSetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!ws->tok_host) {  // one mapped pinned word the kernel writes the argmax to, on first use
    B2D_CUDA(cudaHostAlloc(reinterpret_cast<void**>(&ws->tok_host), 4 * sizeof(int32_t), cudaHostAllocMapped),
             "mapped token word");
    B2D_CUDA(cudaHostGetDevicePointer(reinterpret_cast<void**>(&ws->tok_dev), ws->tok_host, 0),
             "mapped token word address");
  }
  // The token and position travel in the launch's arguments; the kernel
  // writes the argmax straight into the mapped host word.  Every call ends
  // with the stream synchronised, so no earlier step still writes it.
  ws->tok_host[0] = -1;
  b2d_status s = launch_b1(m, ws, nullptr, nullptr, kv_dev, logits_dev, ws->tok_dev, 1, nullptr, st, tok, pos);
  const cudaError_t e = cudaStreamSynchronize(st);  // also on the error path
  if (s != B2D_OK) return s;
  if (e != cudaSuccess) return cuda_fail(e, "sync");
  *next_tok = *reinterpret_cast<volatile int32_t*>(ws->tok_host);
  return B2D_OK;
}

b2d_status b2d_decode_steps(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, const int32_t* pos_dev,
                            int n_steps, void* kv_dev, int32_t* tokens_dev, float* logits_dev, void* stream) {
  if (!m || !ws || ws->m != m || !tok_dev || !pos_dev || !kv_dev || !tokens_dev || n_steps < 1 ||
      n_steps > m->cfg.context_len)
    return B2D_ERR_INVALID_ARG;
  B2D_CUDA(cudaSetDevice(m->device), "cudaSetDevice");
  return launch_b1(m, ws, tok_dev, pos_dev, kv_dev, logits_dev, tokens_dev + (n_steps - 1), n_steps, tokens_dev,
                   static_cast<cudaStream_t>(stream));
}

b2d_status b2d_sample(b2d_ws* ws, const float* logits_dev, int batch, int vocab, const int32_t* history_dev,
                      int hist_cap, const int32_t* hist_len_dev, const double* uniforms_dev,
                      const b2d_sampling* params, int32_t* out_tok_dev, void* stream) {
  if (!ws || !logits_dev || batch < 1 || vocab < 1 || vocab > b2d::kSamplerMaxVocab || !params ||
      !out_tok_dev || hist_cap < 0 || (hist_cap > 0 && (!history_dev || !hist_len_dev)) ||
      !(params->temperature >= 0.0) || !(params->top_p > 0.0) || !(params->rep_penalty > 0.0))
    return B2D_ERR_INVALID_ARG;
  if (params->temperature > 0.0 && !uniforms_dev) return B2D_ERR_INVALID_ARG;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2D_CUDA(cudaSetDevice(ws->m->device), "cudaSetDevice");
  if (params->temperature > 0.0 && params->top_p < 1.0 && batch > ws->sample_rows) {
    // the top-p sort's scratch (256 KB per sequence), grown on first use outside capture
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    B2D_CUDA(cudaStreamIsCapturing(st, &cs), "capture status");
    if (cs != cudaStreamCaptureStatusNone) return B2D_ERR_INVALID_ARG;
    B2D_CUDA(cudaStreamSynchronize(st), "sync");
    cudaFree(ws->sample_scratch);
    ws->sample_scratch = nullptr;
    ws->sample_rows = 0;
    B2D_CUDA(cudaMalloc(&ws->sample_scratch, sizeof(uint64_t) * size_t(batch) * b2d::kSamplerMaxVocab),
             "sampler scratch");
    ws->sample_rows = batch;
  }
  B2D_CUDA(b2d::launch_sampler(logits_dev, batch, vocab, history_dev, hist_cap, hist_len_dev, uniforms_dev,
                               params->temperature, params->top_p, params->rep_penalty, out_tok_dev, st,
                               ws->sample_scratch, ws->sample_trace, ws->sample_mode),
           "sampler launch");
  return B2D_OK;
}

namespace {

b2d_status ensure_weight_maps(b2d_model* m) {
  if (m->maps_ready) return B2D_OK;
  const b2d_config& c = m->cfg;
  const uint64_t D = c.d_model, F = c.d_ff, Q = uint64_t(c.n_heads + 2 * c.n_kv_heads) * 64;
  if (Q % b2d::kGemmBM || D % b2d::kGemmBM || (2 * F) % b2d::kGemmBM || c.vocab_size % b2d::kGemmBM ||
      D % b2d::kGemmBK || F % b2d::kGemmBK || c.n_heads / c.n_kv_heads > 4)  // 4 query heads per attention unit
    return B2D_ERR_UNSUPPORTED;
  CUtensorMap* maps = new (std::nothrow) CUtensorMap[4 * c.n_layers + 1];
  if (!maps) return B2D_ERR_NO_MEMORY;
  bool ok = true;
  for (int l = 0; l < c.n_layers && ok; ++l) {
    const uint8_t* base = m->w + uint64_t(l) * m->lay.layer_stride;
    ok = b2d::make_kmajor_map(&maps[4 * l + 0], base + m->lay.off_qkv, D, Q, b2d::kGemmBM) &&
         b2d::make_kmajor_map(&maps[4 * l + 1], base + m->lay.off_o, D, D, b2d::kGemmBM) &&
         b2d::make_kmajor_map(&maps[4 * l + 2], base + m->lay.off_gu, D, 2 * F, b2d::kGemmBM) &&
         b2d::make_kmajor_map(&maps[4 * l + 3], base + m->lay.off_down, F, D, b2d::kGemmBM);
  }
  ok = ok && b2d::make_kmajor_map(&maps[4 * c.n_layers], m->w + m->lay.off_emb, D, c.vocab_size, b2d::kGemmBM);
  if (!ok) {
    delete[] maps;
    return B2D_ERR_CUDA;
  }
  m->wmaps = maps;
  m->maps_ready = true;
  return B2D_OK;
}

}  // namespace

namespace {

// The batched step's kernel sequence over `batch` rows (tokens `tok`, positions
// `pos`, device arrays).  prefill = false: decode rows of independent
// sequences over a paged pool (`table` [batch][bps]); each row's new K/V is
// appended by the attention kernel.  prefill = true: rows are positions of
// ONE sequence whose cache `cache` is contiguous in the reference layout
// (table = nullptr) or paged (table = its row); the K/V of all rows are
// appended first, per layer.
// logits == nullptr skips the output projection (earlier prefill chunks);
// next_tok == nullptr skips the argmax; out_tail > 0: the output projection
// and the argmax cover only the last out_tail rows, written as rows 0.. .
// table_ld: entries between rows' table rows (default: bps for decode, 0 for
// a prefill, whose rows then share the one table row `table` [bps]).
b2d_status run_rows(b2d_model* m, b2d_ws* ws, const int32_t* tok, const int32_t* pos, int batch, void* cache,
                    const int32_t* table, int bps, int num_blocks, bool prefill, float* logits, int32_t* next_tok,
                    cudaStream_t st, int out_tail = 0, int table_ld = -1) {
  b2d_status s = ensure_weight_maps(m);
  if (s != B2D_OK) return s;
  const b2d_config& c = m->cfg;
  const int D = c.d_model, F = c.d_ff, Q = (c.n_heads + 2 * c.n_kv_heads) * 64, V = c.vocab_size;
  uint32_t* status = &ws->ctl->status;
  const float* ln1 = reinterpret_cast<const float*>(m->w + m->lay.off_ln1);
  const float* ln2 = reinterpret_cast<const float*>(m->w + m->lay.off_ln2);
  const float* lnf = reinterpret_cast<const float*>(m->w + m->lay.off_lnf);
  const __nv_bfloat16* emb = reinterpret_cast<const __nv_bfloat16*>(m->w + m->lay.off_emb);

  const bool pdl = !ws->no_pdl;
  int gl = 0;  // projection launches so far (diagnostic stamps)
  int launches_other = 0;  // embedding, attention, RMSNorm, argmax launches
  b2d::GemmArgs g{};
  auto gemm = [&](const CUtensorMap& wm, const CUtensorMap* xmaps, int epi, const b2d::GemmPlan& pl) {
    g.ksplit = pl.ksplit;
    g.trace = ws->gemm_trace && gl < kTraceLaunches ? ws->gemm_trace + size_t(gl) * kTraceCtas * b2d::kGemmStamps
                                                     : nullptr;
    g.trace_ctas = kTraceCtas;
    ++gl;
    return b2d::launch_gemm(wm, xmaps[bn_index(pl.bn)], g, epi, st, pdl, pl.bn);
  };
  // Layer projections prefer tiles of at most 64 batch rows (more CTAs, a
  // shorter epilogue each); the logits projection up to 256 (fewer re-reads
  // of the 65 MB embedding).
  b2d::GemmPlan p_qkv = b2d::gemm_plan(Q, batch, D, 64), p_o = b2d::gemm_plan(D, batch, D, 64);
  b2d::GemmPlan p_gu = b2d::gemm_plan(2 * F, batch, D, 64), p_dn = b2d::gemm_plan(D, batch, F, 64);
  b2d::GemmPlan p_lg = b2d::gemm_plan(V, batch, D, 256);
  if (ws->force_ksplit) {  // clamped to each projection's K / 64
    const int f = ws->force_ksplit;
    p_qkv.ksplit = std::min(f, D / b2d::kGemmBK);
    p_o.ksplit = std::min(f, D / b2d::kGemmBK);
    p_gu.ksplit = std::min(f, D / b2d::kGemmBK);
    p_dn.ksplit = std::min(f, F / b2d::kGemmBK);
    p_lg.ksplit = std::min(f, D / b2d::kGemmBK);
  }
  const int ss_tiles = D / b2d::kGemmBM;
  B2D_CUDA(launch_k(b2d::embed_rows_kernel, dim3(batch), dim3(256), st, false, emb, tok, V, D, ln1, ws->H, ws->X,
                    ws->ss, ws->rows, ss_tiles, status), "embed");
  ++launches_other;
  g.N = batch;
  g.err = status;
  g.norm_eps = c.rms_eps;
  g.ss_dim = D;
  g.ss_ld = ws->rows;
  b2d::PagedAttnArgs pa{};
  pa.qkv = ws->qkv; pa.pos = pos; pa.pool = static_cast<__nv_bfloat16*>(cache);
  pa.table = table; pa.bps = bps; pa.num_blocks = num_blocks; pa.append = !prefill;
  pa.table_ld = table_ld >= 0 ? table_ld : prefill ? 0 : bps;
  pa.n_heads = c.n_heads; pa.n_kv = c.n_kv_heads; pa.ctx = c.context_len;
  pa.rcos = reinterpret_cast<const float*>(m->w + m->lay.off_cos);
  pa.rsin = reinterpret_cast<const float*>(m->w + m->lay.off_sin);
  pa.out = ws->A; pa.ldo = D; pa.status = status;
  // Paged pool: pages arrive as TMA tensor copies (two 2 KB boxes per page)
  // when the pool's rows of 64 bf16 are addressable with 32-bit coordinates.
  CUtensorMap kvmap{};
  const uint64_t pool_rows = uint64_t(c.n_layers) * uint64_t(num_blocks) * 2 * uint64_t(c.n_kv_heads) * b2d::kPageTokens;
  const bool att_tma = table != nullptr && pool_rows <= 0x7fffffffull;
  if (att_tma) {
    if (ws->kvmap_pool != cache || ws->kvmap_nblk != num_blocks) {
      if (!b2d::make_kmajor_map(&ws->kvmap, cache, 64, pool_rows, b2d::kPageTokens)) return B2D_ERR_CUDA;
      ws->kvmap_pool = cache;
      ws->kvmap_nblk = num_blocks;
    }
    kvmap = ws->kvmap;
  }
  // Units (warps) per (row, kv head) and each unit's page ring (measured at
  // B=256 / 2048, TMA pages):
  //  * rows split while the (row, kv head) pairs alone leave SMs idle, with
  //    6-page rings (8 warps per SM);
  //  * rows left whole by that rule whose split units fit one wave only with
  //    2-page rings (22 warps per SM): split in two with 2-page rings (B=256:
  //    1170 -> 1155 us per step at position 190, 1282 -> 1262 at 300);
  //  * units far beyond the warp slots (a one-wave batch of 2048): 4-page
  //    rings (457k -> 487k tok/s; 6-page rings are faster for waves of 256).
  const int pairs = batch * c.n_kv_heads;
  int att_stages = b2d::kPaStages;
  {
    const int target = 10 * m->grid;
    int sp = ws->force_att_cpc ? ws->force_att_cpc : std::max(1, target / pairs);
    sp = std::min(sp, std::min(b2d::kPaMaxSplits, (c.context_len + 15) / 16));
    pa.cpc = sp >= 4 ? 4 : sp >= 2 ? 2 : 1;  // a row's units share one CTA of pa_warps(splits) warps
    // decode only: prompt rows keep the units of the contiguous-cache path,
    // so a paged prefill equals a contiguous one bit for bit
    if (att_tma && !prefill && pa.cpc == 1 && !ws->force_att_cpc && 2 * pairs > 8 * m->grid &&
        2 * pairs <= 22 * m->grid && c.context_len >= 2 * b2d::kPageTokens) {
      pa.cpc = 2;
      att_stages = b2d::kPaStagesSplit;
    } else if (att_tma && !prefill && pa.cpc == 1 && pairs > 16 * m->grid) {
      att_stages = b2d::kPaStagesShallow;
    }
  }
  const int att_w = b2d::pa_warps(pa.cpc);
  B2D_CUDA(attn_smem_attrs(), "attention attributes");
  const int att_units = pairs * pa.cpc;
  auto* att_k2 = !att_tma ? b2d::paged_attn_mma_kernel<2, false>
                 : att_stages == b2d::kPaStagesSplit ? b2d::paged_attn_mma_kernel<2, true, b2d::kPaStagesSplit>
                 : att_stages == b2d::kPaStagesShallow ? b2d::paged_attn_mma_kernel<2, true, b2d::kPaStagesShallow>
                                                      : b2d::paged_attn_mma_kernel<2, true>;
  auto* att_k4 = att_tma ? b2d::paged_attn_mma_kernel<4, true> : b2d::paged_attn_mma_kernel<4, false>;
  const int att_smem2 = b2d::pa_smem_bytes(2, att_tma, att_stages);
  // RMSNorm of the residual stream, folded: each residual projection writes
  // X = bf16(h * g_next) and per-tile sums of squares; the next projection
  // (qkv, gate/up, logits) scales its result columns by rsqrt(mean + eps).
  for (int l = 0; l < c.n_layers; ++l) {
    // X = bf16(H * ln1[l]) and its statistics come from the embedding (l = 0) or the previous down projection
    g.M = Q; g.K = D; g.y = ws->qkv; g.resid = nullptr; g.ldy = Q;
    g.ss_in = ws->ss; g.xg_out = nullptr; g.xg_gain = nullptr; g.ss_out = nullptr;
    B2D_CUDA(gemm(m->wmaps[4 * l + 0], ws->xmap, b2d::EPI_F32, p_qkv), "qkv");
    pa.layer = l;
    pa.trace = ws->att_trace ? ws->att_trace + size_t(l) * kAttTraceUnits * 8 : nullptr;
    pa.trace_units = kAttTraceUnits;
    if (prefill)  // every row's K/V in the cache before any row attends
      B2D_CUDA(launch_k(b2d::kv_append_kernel, dim3(batch, c.n_kv_heads), dim3(32), st, pdl, pa), "kv append");
    if (att_w == 2)
      B2D_CUDA(launch_k_smem(att_k2, dim3((att_units + 1) / 2), dim3(64), att_smem2, st, pdl, kvmap, pa, batch),
               "attention");
    else
      B2D_CUDA(launch_k_smem(att_k4, dim3((att_units + 3) / 4), dim3(128), b2d::pa_smem_bytes(4, att_tma), st, pdl,
                             kvmap, pa, batch),
               "attention");
    launches_other += prefill ? 2 : 1;
    g.M = D; g.K = D; g.y = ws->Hm; g.resid = ws->H; g.ldy = D;
    g.ss_in = nullptr; g.xg_out = ws->X; g.xg_gain = ln2 + size_t(l) * D; g.ss_out = ws->ss;
    B2D_CUDA(gemm(m->wmaps[4 * l + 1], ws->amap, b2d::EPI_RESID_F32, p_o), "o");
    g.M = 2 * F; g.K = D; g.ybf = ws->ACT; g.ldy = F;
    g.ss_in = ws->ss; g.xg_out = nullptr; g.xg_gain = nullptr; g.ss_out = nullptr;
    B2D_CUDA(gemm(m->wmaps[4 * l + 2], ws->xmap, b2d::EPI_SWIGLU_BF16, p_gu), "gate/up");
    const float* next_g = l + 1 < c.n_layers ? ln1 + size_t(l + 1) * D : lnf;  // next ln1, or the final norm
    g.M = D; g.K = F; g.y = ws->H; g.resid = ws->Hm; g.ldy = D;
    g.ss_in = nullptr; g.xg_out = ws->X; g.xg_gain = next_g; g.ss_out = ws->ss;
    B2D_CUDA(gemm(m->wmaps[4 * l + 3], ws->actmap, b2d::EPI_RESID_F32, p_dn), "down");
  }
  if (logits == nullptr) {  // an earlier prefill chunk: only its cache rows are needed
    ws->last_launches = gl + launches_other;
    return B2D_OK;
  }
  g.M = V; g.K = D; g.y = logits; g.resid = nullptr; g.ldy = V;
  g.ss_in = ws->ss; g.xg_out = nullptr; g.xg_gain = nullptr; g.ss_out = nullptr;
  const int n_out = out_tail > 0 ? out_tail : batch;
  if (out_tail > 0) {
    g.N = n_out;
    g.n_base = batch - n_out;
    p_lg = b2d::gemm_plan(V, n_out, D, 256);
  }
  B2D_CUDA(gemm(m->wmaps[4 * c.n_layers], ws->xmap, b2d::EPI_F32, p_lg), "logits");
  g.N = batch;
  g.n_base = 0;
  if (next_tok) {
    B2D_CUDA(launch_k(b2d::argmax_rows_kernel, dim3(n_out), dim3(1024), st, pdl, (const float*)logits, V, V,
                      next_tok), "argmax");
    ++launches_other;
  }
  ws->last_launches = gl + launches_other;
  return B2D_OK;
}

}  // namespace

b2d_status b2d_decode_step_paged(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, const int32_t* pos_dev,
                                 int batch, void* kv_pool_dev, const int32_t* block_table_dev,
                                 int blocks_per_seq, int num_blocks, float* logits_dev, int32_t* next_tok_dev,
                                 void* stream) {
  if (!m || !ws || ws->m != m || !tok_dev || !pos_dev || !kv_pool_dev || !block_table_dev || !next_tok_dev ||
      batch < 1 || batch > ws->max_batch || ws->max_batch < 2 || blocks_per_seq < 1 || num_blocks < 1)
    return B2D_ERR_INVALID_ARG;
  B2D_CUDA(cudaSetDevice(m->device), "cudaSetDevice");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  float* lg = logits_dev ? logits_dev : ws->logits;
  // The step is ~5 x n_layers dependent launches; from the second call with
  // the same arguments on, it is replayed from a CUDA graph (one host call).
  // Direct launches when graphs are off or the caller's stream is capturing
  // (its own capture then records the kernels).
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (!ws->no_graph && cudaStreamIsCapturing(st, &cs) == cudaSuccess && cs == cudaStreamCaptureStatusNone) {
    const void* key[6] = {tok_dev, pos_dev, kv_pool_dev, block_table_dev, lg, next_tok_dev};
    b2d_ws::StepGraph* g = nullptr;
    for (auto& c : ws->graphs)
      if (c.uses > 0 && std::equal(key, key + 6, c.ptr) && c.batch == batch && c.bps == blocks_per_seq &&
          c.nblk == num_blocks && c.tune == ws->tune_gen) {
        g = &c;
        break;
      }
    if (!g) {  // least recently used entry
      g = &ws->graphs[0];
      for (auto& c : ws->graphs)
        if (c.tick < g->tick) g = &c;
      if (g->exec) cudaGraphExecDestroy(g->exec);
      *g = b2d_ws::StepGraph{};
      std::copy(key, key + 6, g->ptr);
      g->batch = batch; g->bps = blocks_per_seq; g->nblk = num_blocks; g->tune = ws->tune_gen;
    }
    g->tick = ++ws->graph_tick;
    if (g->uses++ > 0) {  // seen before: capture once (on a private stream; nothing runs), then replay
      if (!g->exec) {
        if (!ws->cap_stream) B2D_CUDA(cudaStreamCreateWithFlags(&ws->cap_stream, cudaStreamNonBlocking), "stream");
        B2D_CUDA(cudaStreamBeginCapture(ws->cap_stream, cudaStreamCaptureModeThreadLocal), "begin capture");
        b2d_status s = run_rows(m, ws, tok_dev, pos_dev, batch, kv_pool_dev, block_table_dev, blocks_per_seq,
                                num_blocks, false, lg, next_tok_dev, ws->cap_stream);
        cudaGraph_t graph = nullptr;
        const cudaError_t e = cudaStreamEndCapture(ws->cap_stream, &graph);
        if (s == B2D_OK && e != cudaSuccess) s = cuda_fail(e, "end capture");
        if (s == B2D_OK) {
          const cudaError_t ei = cudaGraphInstantiate(&g->exec, graph, 0);
          if (ei != cudaSuccess) {
            g->exec = nullptr;
            s = cuda_fail(ei, "graph instantiate");
          }
        }
        if (graph) cudaGraphDestroy(graph);
        if (s != B2D_OK) {
          g->uses = 0;
          return s;
        }
        g->launches = ws->last_launches;
      }
      ws->last_launches = g->launches;
      B2D_CUDA(cudaGraphLaunch(g->exec, st), "graph launch");
      return B2D_OK;
    }
  }
  return run_rows(m, ws, tok_dev, pos_dev, batch, kv_pool_dev, block_table_dev, blocks_per_seq, num_blocks, false,
                  lg, next_tok_dev, st);
}

namespace {

// Prompt positions start_pos.. of one sequence through run_rows, up to
// kPrefillRows per chunk; `table` = nullptr: `cache` is that sequence's
// contiguous cache, else the paged pool and `table` its block-table row.
b2d_status prefill_rows(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, int n_tokens, int start_pos, void* cache,
                        const int32_t* table, int bps, int num_blocks, float* logits_dev, int32_t* next_tok_dev,
                        cudaStream_t st) {
  B2D_CUDA(cudaSetDevice(m->device), "cudaSetDevice");
  const int V = m->cfg.vocab_size;
  for (int c0 = 0; c0 < n_tokens; c0 += kPrefillRows) {
    const int rows = std::min(kPrefillRows, n_tokens - c0);
    const bool last = c0 + rows == n_tokens;
    B2D_CUDA(launch_k(iota_kernel, dim3((rows + 127) / 128), dim3(128), st, !ws->no_pdl, ws->prefill_pos,
                      start_pos + c0, rows), "positions");
    b2d_status s = run_rows(m, ws, tok_dev + c0, ws->prefill_pos, rows, cache, table, bps, num_blocks, true,
                            last && (logits_dev || next_tok_dev) ? ws->logits : nullptr, nullptr, st, 1);
    if (s != B2D_OK) return s;
    if (last) {
      const float* lrow = ws->logits;  // the last position's logits (row 0)
      if (logits_dev)
        B2D_CUDA(cudaMemcpyAsync(logits_dev, lrow, sizeof(float) * V, cudaMemcpyDeviceToDevice, st), "logits row");
      if (next_tok_dev)
        B2D_CUDA(launch_k(b2d::argmax_rows_kernel, dim3(1), dim3(1024), st, false, lrow, V, V, next_tok_dev),
                 "argmax");
    }
  }
  return B2D_OK;
}

}  // namespace

b2d_status b2d_prefill(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, int n_tokens, int start_pos, void* kv_dev,
                       float* logits_dev, int32_t* next_tok_dev, void* stream) {
  if (!m || !ws || ws->m != m || !tok_dev || !kv_dev || n_tokens < 1 || start_pos < 0 ||
      start_pos + n_tokens > m->cfg.context_len)
    return B2D_ERR_INVALID_ARG;
  return prefill_rows(m, ws, tok_dev, n_tokens, start_pos, kv_dev, nullptr, 0, 0, logits_dev, next_tok_dev,
                      static_cast<cudaStream_t>(stream));
}

b2d_status b2d_prefill_paged(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, int n_tokens, int start_pos,
                             void* kv_pool_dev, const int32_t* table_row_dev, int blocks_per_seq, int num_blocks,
                             float* logits_dev, int32_t* next_tok_dev, void* stream) {
  if (!m || !ws || ws->m != m || !tok_dev || !kv_pool_dev || !table_row_dev || n_tokens < 1 || start_pos < 0 ||
      blocks_per_seq < 1 || num_blocks < 1 || start_pos + n_tokens > m->cfg.context_len ||
      start_pos + n_tokens > blocks_per_seq * b2d::kPageTokens)
    return B2D_ERR_INVALID_ARG;
  return prefill_rows(m, ws, tok_dev, n_tokens, start_pos, kv_pool_dev, table_row_dev, blocks_per_seq, num_blocks,
                      logits_dev, next_tok_dev, static_cast<cudaStream_t>(stream));
}

b2d_status b2d_prefill_rows(b2d_model* m, b2d_ws* ws, const int32_t* tok_dev, const int32_t* pos_dev, int n_rows,
                            void* kv_pool_dev, const int32_t* table_dev, int blocks_per_seq, int num_blocks,
                            int n_out, float* logits_dev, int32_t* next_tok_dev, void* stream) {
  if (!m || !ws || ws->m != m || !tok_dev || !pos_dev || !kv_pool_dev || !table_dev || n_rows < 1 ||
      n_rows > kPrefillRows || blocks_per_seq < 1 || num_blocks < 1 || n_out < 0 || n_out > n_rows ||
      (n_out == 0 && (logits_dev || next_tok_dev)))
    return B2D_ERR_INVALID_ARG;
  B2D_CUDA(cudaSetDevice(m->device), "cudaSetDevice");
  float* lg = n_out == 0 || (!logits_dev && !next_tok_dev) ? nullptr : logits_dev ? logits_dev : ws->logits;
  return run_rows(m, ws, tok_dev, pos_dev, n_rows, kv_pool_dev, table_dev, blocks_per_seq, num_blocks, true, lg,
                  next_tok_dev, static_cast<cudaStream_t>(stream), n_out, blocks_per_seq);
}

int b2d_prefill_rows_max(void) { return kPrefillRows; }

int b2d_batched_launches(const b2d_ws* ws) { return ws ? ws->last_launches : 0; }

// Test hook: Y = X . W^T on the tensor-core GEMM with the chosen epilogue.
b2d_status b2d_test_gemm(const void* w_dev, int M, int K, const void* x_dev, int N, int epi, float* y_dev,
                         const float* resid_dev, void* ybf_dev, int ldy, void* stream) {
  int ks = epi >> 8;
  epi &= 0xff;
  if (!w_dev || !x_dev || M <= 0 || K <= 0 || N <= 0 || M % b2d::kGemmBM || K % b2d::kGemmBK || epi < 0 ||
      epi > 2 || ldy <= 0 || ks < 0 || ks > b2d::kGemmMaxSplit || ks > K / b2d::kGemmBK || (epi != b2d::EPI_SWIGLU_BF16 && !y_dev) || (epi == b2d::EPI_RESID_F32 && !resid_dev) ||
      (epi == b2d::EPI_SWIGLU_BF16 && !ybf_dev))
    return B2D_ERR_INVALID_ARG;
  static uint32_t* err = nullptr;
  if (!err) B2D_CUDA(cudaMalloc(&err, sizeof(uint32_t)), "err word");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  B2D_CUDA(cudaMemsetAsync(err, 0, sizeof(uint32_t), st), "clear err");
  CUtensorMap wm, xm;
  if (!b2d::make_kmajor_map(&wm, w_dev, K, M, b2d::kGemmBM) ||
      !b2d::make_kmajor_map(&xm, x_dev, K, N, b2d::gemm_bn_for(N)))
    return B2D_ERR_INVALID_ARG;
  b2d::GemmArgs g{};
  g.M = M; g.N = N; g.K = K;
  g.y = y_dev; g.resid = resid_dev; g.ybf = static_cast<__nv_bfloat16*>(ybf_dev); g.ldy = ldy; g.err = err;
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, 0);
  g.ksplit = ks ? ks : b2d::gemm_ksplit_for(M, N, K, sms);
  B2D_CUDA(b2d::launch_gemm(wm, xm, g, epi, st, false, b2d::gemm_bn_for(N)), "gemm launch");
  uint32_t h = 0;
  B2D_CUDA(cudaMemcpyAsync(&h, err, sizeof(h), cudaMemcpyDeviceToHost, st), "read err");
  B2D_CUDA(cudaStreamSynchronize(st), "sync");
  return h ? B2D_ERR_DEVICE_TIMEOUT : B2D_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Decode step without any allocation (b2d_decode_step_static).
//
// Some callers cannot allocate device memory at all: a host that hands this
// library only the buffers it owns (an inference server or plugin host with
// its own device-memory pool), or code running where cudaMalloc is not
// allowed.  For them the exchange words, control words and argmax partials
// that b2d_workspace_create would allocate live in one fixed array in device
// memory, defined here at file scope.  The array is b2d::kStaticScratchBytes
// (4 MiB) long, and every GPU that loads this library holds it until the
// process exits.
//
// Host code must not hand `g_static_scratch` itself to a kernel: in host code
// that name is a host-side stand-in, not a device address.  The device address
// is looked up once per device with cudaGetSymbolAddress (with that device
// current) on the first call made on that device, so make that first call
// before any stream capture.  Every call reuses the same array and finds in it
// whatever the previous call left: each call therefore clears the area it uses
// (a stream-ordered memset) before its launch.  Calls that overlap on the GPU
// (other streams, other threads) race on the array; keep them ordered.
// ---------------------------------------------------------------------------
namespace b2d {
constexpr size_t kStaticScratchBytes = size_t(4) << 20;
constexpr size_t kStaticCtlOffset = 0;          // Control (640 B)
constexpr size_t kStaticArgmaxOffset = 1024;    // am_val[kStaticMaxGrid], am_idx[kStaticMaxGrid]
constexpr int kStaticMaxGrid = 1024;
constexpr size_t kStaticWordsOffset = 16384;    // exchange words
static_assert(sizeof(Control) <= kStaticArgmaxOffset - kStaticCtlOffset, "control block");
static_assert(kStaticArgmaxOffset + 8 * kStaticMaxGrid <= kStaticWordsOffset, "argmax partials");
}  // namespace b2d

static __device__ __align__(256) unsigned char g_static_scratch[b2d::kStaticScratchBytes];

namespace {

struct StaticDeviceState {
  bool ready;
  unsigned char* scratch;  // device address of g_static_scratch on this device
  int sms;
  int smem_set;            // bitmask of shape ops whose smem attribute is set
  int c_grid[8];           // per shape ops: the cluster kernel's grid (0 = flat kernel)
};
constexpr int kMaxDevices = 64;
StaticDeviceState g_static_dev[kMaxDevices];
std::mutex g_static_mu;

// Looks up g_static_scratch's device address on `device` (current) once.
// The caller holds g_static_mu.
b2d_status static_lookup(int device, StaticDeviceState& st) {
  if (!st.ready) {
    void* p = nullptr;
    B2D_CUDA(cudaGetSymbolAddress(&p, g_static_scratch), "cudaGetSymbolAddress(g_static_scratch)");
    if (p == nullptr) return cuda_fail(cudaErrorInvalidSymbol, "cudaGetSymbolAddress(g_static_scratch)");
    int sms = 0, coop = 0;
    B2D_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device), "sm count");
    B2D_CUDA(cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device), "coop attr");
    if (!coop) return B2D_ERR_LAUNCH;
    if (sms < b2d::kMinGrid || sms > b2d::kStaticMaxGrid) return B2D_ERR_UNSUPPORTED;
    st.scratch = static_cast<unsigned char*>(p);
    st.sms = sms;
    st.ready = true;
  }
  return B2D_OK;
}

b2d_status static_setup(int device, const ShapeOps* ops, int ops_index, StaticDeviceState** out) {
  std::lock_guard<std::mutex> lock(g_static_mu);
  StaticDeviceState& st = g_static_dev[device];
  b2d_status s = static_lookup(device, st);
  if (s != B2D_OK) return s;
  if (!(st.smem_set & (1 << ops_index))) {
    B2D_CUDA(cudaFuncSetAttribute(ops->kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(ops->smem)),
             "cudaFuncSetAttribute(smem)");
    B2D_CUDA(cudaFuncSetAttribute(ops->kernel_c, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  static_cast<int>(ops->smem_c)),
             "cudaFuncSetAttribute(smem)");
    st.c_grid[ops_index] = b1c_grid(ops);
    st.smem_set |= 1 << ops_index;
  }
  *out = &st;
  return B2D_OK;
}

}  // namespace

extern "C" b2d_status b2d_decode_step_static(const b2d_config* cfg, const void* weights_dev,
                                             uint64_t weights_bytes, const int32_t* tok_dev,
                                             const int32_t* pos_dev, void* kv_dev, float* logits_dev,
                                             int32_t* next_tok_dev, void* stream) {
  if (!config_valid(cfg) || !weights_dev || (reinterpret_cast<uintptr_t>(weights_dev) & 255u) || !tok_dev ||
      !pos_dev || !kv_dev || !next_tok_dev)
    return B2D_ERR_INVALID_ARG;
  const ShapeOps* ops = find_ops(cfg);
  if (!ops) return B2D_ERR_UNSUPPORTED;
  b2d_weights_layout_t lay;
  compute_layout(cfg, &lay);
  if (weights_bytes < lay.total_bytes) return B2D_ERR_INVALID_ARG;
  // Exchange-word layout, as b2d_workspace_create lays it out.
  const uint32_t qkv = uint32_t(cfg->n_heads + 2 * cfg->n_kv_heads) * 64;
  const uint32_t w_att = uint32_t(cfg->d_model) + qkv;
  const uint32_t w_hm = w_att + uint32_t(cfg->n_heads) * b2d::kMaxSplits * b2d::kAttWords;
  const uint32_t w_act = w_hm + uint32_t(cfg->d_model);
  const uint32_t layer_words = (w_act + uint32_t(cfg->d_ff) + 1) & ~1u;
  const size_t n_words = size_t(cfg->n_layers) * layer_words + cfg->d_model;
  // The flat kernel uses exchange words, the cluster kernel residual
  // accumulators: whichever runs takes the area after the argmax partials.
  const size_t words_bytes = n_words * sizeof(uint64_t);
  const size_t acc_bytes = size_t(2) * 2 * cfg->n_layers * cfg->d_model * b2d::kAccStride * sizeof(uint64_t);
  // refused before any device work when neither kernel's area fits
  if (b2d::kStaticWordsOffset + std::min(words_bytes, acc_bytes) > b2d::kStaticScratchBytes)
    return B2D_ERR_SCRATCH_LIMIT;
  int device = 0;
  B2D_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) return B2D_ERR_UNSUPPORTED;
  // Every buffer must be device memory of the current device: this entry
  // point serves hosts with their own memory pools, where a host pointer or
  // another GPU's buffer is an easy mistake that would otherwise reach the
  // kernel unchecked.
  const void* bufs[] = {weights_dev, tok_dev, pos_dev, kv_dev, next_tok_dev, logits_dev};
  for (const void* b : bufs) {
    if (b == nullptr) continue;  // only logits_dev may be null (checked above)
    cudaPointerAttributes pa;
    B2D_CUDA(cudaPointerGetAttributes(&pa, b), "cudaPointerGetAttributes");
    if (pa.type != cudaMemoryTypeDevice || pa.device != device) return B2D_ERR_INVALID_ARG;
  }
  StaticDeviceState* st = nullptr;
  const int ops_index = ops->d == 1024 ? 0 : 1;
  b2d_status s = static_setup(device, ops, ops_index, &st);
  if (s != B2D_OK) return s;
  const int c_grid = st->c_grid[ops_index];
  const size_t used = b2d::kStaticWordsOffset + (c_grid > 0 ? acc_bytes : words_bytes);
  if (used > b2d::kStaticScratchBytes) return B2D_ERR_SCRATCH_LIMIT;
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  // Everything this call reads before writing starts from zero.
  B2D_CUDA(cudaMemsetAsync(st->scratch, 0, used, cs), "clear static scratch");
  const uint8_t* w = static_cast<const uint8_t*>(weights_dev);
  b2d::DecodeArgs A;
  std::memset(&A, 0, sizeof(A));
  A.wbase = w;
  A.layer_stride = lay.layer_stride;
  A.off_qkv = lay.off_qkv;
  A.off_o = lay.off_o;
  A.off_gu = lay.off_gu;
  A.off_down = lay.off_down;
  A.off_emb = lay.off_emb;
  A.ln1 = reinterpret_cast<const float*>(w + lay.off_ln1);
  A.ln2 = reinterpret_cast<const float*>(w + lay.off_ln2);
  A.lnf = reinterpret_cast<const float*>(w + lay.off_lnf);
  A.rcos = reinterpret_cast<const float*>(w + lay.off_cos);
  A.rsin = reinterpret_cast<const float*>(w + lay.off_sin);
  A.tok = tok_dev;
  A.pos = pos_dev;
  A.kv = static_cast<__nv_bfloat16*>(kv_dev);
  A.logits = logits_dev;
  A.next_tok = next_tok_dev;
  A.words = reinterpret_cast<uint64_t*>(st->scratch + b2d::kStaticWordsOffset);
  A.acc = reinterpret_cast<uint64_t*>(st->scratch + b2d::kStaticWordsOffset);
  A.ctl = reinterpret_cast<b2d::Control*>(st->scratch + b2d::kStaticCtlOffset);
  A.am_val = reinterpret_cast<float*>(st->scratch + b2d::kStaticArgmaxOffset);
  A.am_idx = reinterpret_cast<int32_t*>(st->scratch + b2d::kStaticArgmaxOffset + 4 * b2d::kStaticMaxGrid);
  A.layer_words = layer_words;
  A.w_att = w_att;
  A.w_hm = w_hm;
  A.w_act = w_act;
  A.vocab = cfg->vocab_size;
  A.n_layers = cfg->n_layers;
  A.ctx = cfg->context_len;
  A.att_T = 128 * ((cfg->context_len + 511) / 512);
  A.grid_part = c_grid > 0 ? c_grid : st->sms;
  A.wait_ns = 2000000000ull;
  A.eps = cfg->rms_eps;
  A.max_inflight = 4;
  if (c_grid > 0) {
    b2d::MapsC maps;  // encoded on the host per call: no allocation
    if (!make_b1c_maps(cfg, ops, w, lay, &maps)) return B2D_ERR_INVALID_ARG;
    B2D_CUDA(launch_b1c(ops->kernel_c, c_grid, ops->smem_c, cs, maps, A), "static decode launch");
    return B2D_OK;
  }
  void* args[] = {&A};
  B2D_CUDA(cudaLaunchCooperativeKernel(ops->kernel, dim3(st->sms), dim3(b2d::kThreads), args, ops->smem, cs),
           "static decode launch");
  return B2D_OK;
}

// Status of the last b2d_decode_step_static call on the current device: the
// control block in the fixed array holds the kernel's status word (a bounded
// wait that ran out, a token or position out of range read on the device).
// Each static call clears that block before its launch, so this reports the
// most recent call only.  Synchronises `stream` first; allocates nothing.
extern "C" b2d_status b2d_static_last_error(void* stream, uint32_t* detail) {
  if (detail) *detail = 0;
  int device = 0;
  B2D_CUDA(cudaGetDevice(&device), "cudaGetDevice");
  if (device < 0 || device >= kMaxDevices) return B2D_ERR_UNSUPPORTED;
  unsigned char* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_static_mu);
    b2d_status s = static_lookup(device, g_static_dev[device]);
    if (s != B2D_OK) return s;
    scratch = g_static_dev[device].scratch;
  }
  cudaStream_t cs = static_cast<cudaStream_t>(stream);
  uint32_t s = 0;
  const b2d::Control* ctl = reinterpret_cast<const b2d::Control*>(scratch + b2d::kStaticCtlOffset);
  B2D_CUDA(cudaMemcpyAsync(&s, &ctl->status, sizeof(s), cudaMemcpyDeviceToHost, cs), "read static status");
  B2D_CUDA(cudaStreamSynchronize(cs), "cudaStreamSynchronize");
  if (detail) *detail = s;
  if (s == 0) return B2D_OK;
  if ((s & 0xF00u) == b2d::ST_TIMEOUT) return B2D_ERR_DEVICE_TIMEOUT;
  if ((s & 0xF00u) == b2d::ST_BAD_INPUT) return B2D_ERR_DEVICE_INPUT;
  return B2D_ERR_DEVICE_HALTED;
}
