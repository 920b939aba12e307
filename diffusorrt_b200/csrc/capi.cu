// Native runtime behind the C ABI in include/diffusorrt_b200.h: model weights, per-request
// sessions (K/V cache, activations, CUDA graphs), and the kernel-level entry points.
//
// One process per GPU; a model and its sessions live on the device given at creation. All
// device work of a session runs on the session's own stream; kernels are chained with
// programmatic dependent launch so each kernel's weight prefetch overlaps its predecessor.
#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/diffusorrt_b200.h"
#include "attention.cuh"
#include "attention_decode.cuh"
#include "common.cuh"
#include "dream.cuh"
#include "gemm.cuh"
#include "gemm_decode.cuh"
#include "gemm_streamk.cuh"
#include "policy.cuh"
#include "quant.cuh"
#include "rowops.cuh"
#include "selector.cuh"

using namespace drt;

// ======================================================================= errors
namespace {
thread_local std::string g_last_error;

int set_error(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}
}  // namespace

#define CK(expr)                                                                                         \
  do {                                                                                                   \
    cudaError_t _e = (expr);                                                                             \
    if (_e != cudaSuccess)                                                                               \
      return set_error(DRT_INTERNAL_ERROR, "%s failed: %s (%s:%d)", #expr, cudaGetErrorString(_e), __FILE__, \
                       __LINE__);                                                                        \
  } while (0)
#define TRY(expr)                 \
  do {                            \
    int _r = (expr);              \
    if (_r != DRT_OK) return _r;  \
  } while (0)
#define REQUIRE(cond, ...)                                     \
  do {                                                         \
    if (!(cond)) return set_error(DRT_INVALID_ARGUMENT, __VA_ARGS__); \
  } while (0)

// ======================================================================= TMA descriptors
namespace {
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// bf16 tensor map with 128-byte swizzle; dims/strides innermost first (strides: rank-1 entries).
int make_map(CUtensorMap* map, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
             const uint32_t* box) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(DRT_INTERNAL_ERROR, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0) return set_error(DRT_INTERNAL_ERROR, "tensor map base not 16-byte aligned");
  cuuint64_t d[3], s[2];
  cuuint32_t b[3], e[3] = {1, 1, 1};
  for (int i = 0; i < rank; ++i) { d[i] = dims[i]; b[i] = box[i]; }
  for (int i = 0; i < rank - 1; ++i) {
    s[i] = strides[i];
    if (s[i] % 16 != 0) return set_error(DRT_INTERNAL_ERROR, "tensor map stride not a multiple of 16 bytes");
  }
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, rank, const_cast<void*>(base), d, s, b, e,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DRT_INTERNAL_ERROR, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return DRT_OK;
}

// Row-major bf16 matrix [rows][cols], box {64 cols, box_rows rows}.
int map_matrix(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  const uint64_t dims[2] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows)};
  const uint64_t strides[1] = {static_cast<uint64_t>(cols) * 2};
  const uint32_t box[2] = {64, static_cast<uint32_t>(box_rows)};
  return make_map(map, base, 2, dims, strides, box);
}

// Row-major uint8 matrix [rows][cols_bytes] (packed quantized weights), box {box_cols bytes, box_rows},
// no swizzle: a box lands as box_rows contiguous rows of box_cols bytes.
int map_u8(CUtensorMap* map, const void* base, int64_t rows, int64_t cols_bytes, int box_cols, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (fn == nullptr) return set_error(DRT_INTERNAL_ERROR, "cuTensorMapEncodeTiled is unavailable");
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0 || cols_bytes % 16 != 0 || box_cols % 16 != 0)
    return set_error(DRT_INTERNAL_ERROR, "packed weight map alignment");
  cuuint64_t d[2] = {static_cast<cuuint64_t>(cols_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t st[1] = {static_cast<cuuint64_t>(cols_bytes)};
  cuuint32_t b[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)}, e[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), d, st, b, e, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(DRT_INTERNAL_ERROR, "cuTensorMapEncodeTiled (u8) failed (%d)", static_cast<int>(r));
  return DRT_OK;
}

thread_local int64_t g_launches = 0;  // kernels enqueued by this thread (launch accounting)

// Launch with optional programmatic dependent launch and a cluster of `cluster_z` CTAs along z.
template <typename Kern, typename... Args>
cudaError_t launch_kc(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, int cluster_z,
                      Args... args) {
  ++g_launches;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pdl) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  if (cluster_z > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 1;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = static_cast<unsigned>(cluster_z);
    ++n;
  }
  cfg.attrs = n ? attr : nullptr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// Launch with programmatic dependent launch and a cluster of `cluster_x` CTAs along x.
template <typename Kern, typename... Args>
cudaError_t launch_cx(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster_x, Args... args) {
  ++g_launches;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster_x > 1) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = static_cast<unsigned>(cluster_x);
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <typename Kern, typename... Args>
cudaError_t launch_k(Kern kernel, dim3 grid, dim3 block, size_t smem, cudaStream_t stream, bool pdl, Args... args) {
  return launch_kc(kernel, grid, block, smem, stream, pdl, 1, args...);
}

int g_num_sms_cache[64] = {0};
int num_sms(int device) {
  if (device < 0 || device >= 64) return 148;
  if (g_num_sms_cache[device] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    g_num_sms_cache[device] = n > 0 ? n : 148;
  }
  return g_num_sms_cache[device];
}

int configure_kernels() {
  static int result = -1;
  static std::once_flag once;
  std::call_once(once, [] {
    result = DRT_OK;
    if (cudaFuncSetAttribute(gemm_swapab_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_swapab_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_swapab_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_swapab_kernel<128, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_streamk_kernel<128, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_streamk_kernel<64, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
        cudaFuncSetAttribute(attn_prefix_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kAttnSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_wide_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kAttnSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(sel_topp_entropy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kToppSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_swapab_kernel<64>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_swapab_kernel<128>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaFuncSetAttribute(attn_prefix_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kDaSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess ||
        cudaFuncSetAttribute(gemm_lm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess)
      result = DRT_INTERNAL_ERROR;
    for (int qb = 0; qb <= 8 && result == DRT_OK; qb += 4)
    for (int epi = 0; epi <= EPI_QKV && result == DRT_OK; ++epi)
      for (int sp = 1; sp <= 16 && result == DRT_OK; sp *= 2) {
        DecGemmKernel k = dec_gemm_kernel(epi, sp, qb);
        if (k == nullptr || cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024) != cudaSuccess ||
            cudaFuncSetAttribute(k, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
          result = DRT_INTERNAL_ERROR;
      }
  });
  if (result != DRT_OK) return set_error(DRT_INTERNAL_ERROR, "cudaFuncSetAttribute failed: %s", cudaGetErrorString(cudaGetLastError()));
  return DRT_OK;
}


constexpr double kTieRel = 9.094947017729282e-13;  // 2^-40
}  // namespace

// ======================================================================= model
// Quantized copy of one linear weight [n][K] (quant.cuh): 4-bit affine (packed nibbles [n][K / 2]) or
// int8 weight-only (bytes [n][K]), bf16 scale and bias [n][K / 64], and the TMA map over the packed
// bytes (box: 64 inputs x 128 rows).
struct QuantW {
  uint8_t* q = nullptr;
  __nv_bfloat16* scale = nullptr;
  __nv_bfloat16* bias = nullptr;
  int bits_cap = 0;  // widest format the packed buffer holds
  CUtensorMap map;
};

struct LayerW {
  __nv_bfloat16 *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
  float *in_norm = nullptr, *post_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr, *bqkv = nullptr;
  CUtensorMap m_qkv, m_o, m_gu, m_down;
  QuantW q_qkv, q_o, q_gu, q_down;
};

struct drt_model {
  drt_model_config cfg;
  int device = 0;
  int H = 0, nq = 0, nkv = 0, I = 0, V = 0, L = 0, rep = 0, tile_pos = 0;
  int qkv_rows = 0, gu_rows = 0;
  std::vector<void*> allocs;
  __nv_bfloat16* embed = nullptr;
  __nv_bfloat16* lm_head = nullptr;
  float* final_norm = nullptr;
  std::vector<LayerW> layers;
  CUtensorMap m_lm;
  bool quantized = false;   // layer linears and lm_head run from their quantized copies
  int qbits = 0;            // 4 (4-bit affine) or 8 (int8 weight-only) when quantized
  QuantW q_lm;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  int rope_pos = 0;
  int64_t bytes = 0;
  // tensor parallelism: this model holds one rank's shard (nq, nkv, I above are the local counts)
  drt_tp_shard shard = {0, 1, 0, 0, 0, 0, 0, 0};
  int nq_full = 0, nkv_full = 0, I_full = 0;
  ncclComm_t comm = nullptr;
};

namespace {
template <typename T>
int dalloc(drt_model* m, T** p, size_t count) {
  void* q = nullptr;
  CK(cudaMalloc(&q, std::max<size_t>(count * sizeof(T), 256)));
  m->allocs.push_back(q);
  m->bytes += static_cast<int64_t>(count * sizeof(T));
  *p = static_cast<T*>(q);
  return DRT_OK;
}

// NCCL, resolved at run time from the process's libnccl.so.2 (the one torch.distributed loaded,
// when it did), so the library carries no link-time NCCL dependency.
struct NcclApi {
  bool ok = false;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
};

int nccl_api(const NcclApi** out) {
  static NcclApi api;
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  if (!api.ok) {
    const char* env = getenv("DRT_NCCL_LIBRARY");
    void* h = nullptr;
    if (env != nullptr && *env) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (h == nullptr) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h == nullptr) return set_error(DRT_UNSUPPORTED, "NCCL not found (libnccl.so.2): %s", dlerror());
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.all_reduce = reinterpret_cast<decltype(api.all_reduce)>(dlsym(h, "ncclAllReduce"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    if (!api.get_unique_id || !api.comm_init_rank || !api.all_reduce || !api.comm_destroy || !api.error_string)
      return set_error(DRT_UNSUPPORTED, "NCCL library lacks an entry point");
    api.ok = true;
  }
  *out = &api;
  return DRT_OK;
}

#define NCCL_CK(api, call)                                                                                   \
  do {                                                                                                       \
    ncclResult_t r_ = (call);                                                                                \
    if (r_ != ncclSuccess) return set_error(DRT_INTERNAL_ERROR, "NCCL: %s", (api)->error_string(r_));      \
  } while (0)

// Megatron-style shard of one rank: attention heads grouped by K/V head, MLP intermediate columns
// in 64-column units (one SwiGLU tile pairs 64 gate and 64 up rows).
int tp_geometry(const drt_model_config* cfg, int rank, int world, drt_tp_shard* out) {
  REQUIRE(world >= 1 && rank >= 0 && rank < world, "rank %d outside a group of %d", rank, world);
  const int nq = cfg->attention_heads, nkv = cfg->num_kv_heads;
  REQUIRE(nkv > 0 && nq % nkv == 0, "attention_heads must divide by num_kv_heads");
  const int rep = nq / nkv;
  drt_tp_shard g;
  g.rank = rank;
  g.world = world;
  if (nkv % world == 0) {
    g.kv_heads = nkv / world;
    g.kv_head0 = rank * g.kv_heads;
    g.q_heads = g.kv_heads * rep;
    g.q_head0 = g.kv_head0 * rep;
  } else if (world % nkv == 0 && world / nkv <= rep) {
    // several ranks per K/V head: each projects that head and takes a share of its query heads
    const int per = world / nkv, j = rank % per;
    g.kv_heads = 1;
    g.kv_head0 = rank / per;
    g.q_heads = rep / per + (j < rep % per ? 1 : 0);
    g.q_head0 = g.kv_head0 * rep + j * (rep / per) + std::min(j, rep % per);
  } else {
    return set_error(DRT_UNSUPPORTED, "%d ranks do not shard %d K/V heads", world, nkv);
  }
  REQUIRE(cfg->intermediate_size % 64 == 0, "intermediate_size must be a multiple of 64");
  const int units = cfg->intermediate_size / 64;
  REQUIRE(units >= world, "intermediate_size too small for %d ranks", world);
  const int u = units / world, extra = units % world;
  g.inter = 64 * (u + (rank < extra ? 1 : 0));
  g.inter0 = 64 * (rank * u + std::min(rank, extra));
  *out = g;
  return DRT_OK;
}

int fill_f32(float* p, int64_t n, float v, cudaStream_t st) {
  fill_f32_kernel<<<static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4096)), 256, 0, st>>>(p, n, v);
  CK(cudaGetLastError());
  return DRT_OK;
}

// Host RoPE tables in the reference's float32 arithmetic (mlx_forward.py:1566-1595); used when
// the caller does not install tables of its own.
void host_rope(std::vector<float>& c, std::vector<float>& s, int n_pos, float theta) {
  c.resize(static_cast<size_t>(n_pos) * 64);
  s.resize(static_cast<size_t>(n_pos) * 64);
  for (int i = 0; i < 64; ++i) {
    const float expo = static_cast<float>(i) / 64.0f;
    const float inv = 1.0f / powf(theta, expo);
    for (int p = 0; p < n_pos; ++p) {
      const float f = static_cast<float>(p) * inv;
      c[static_cast<size_t>(p) * 64 + i] = cosf(f);
      s[static_cast<size_t>(p) * 64 + i] = sinf(f);
    }
  }
}

int parse_layer_key(const char* key, int* layer, std::string* rest) {
  const char* pre = "model.layers.";
  if (strncmp(key, pre, strlen(pre)) != 0) return 0;
  const char* p = key + strlen(pre);
  char* end = nullptr;
  long l = strtol(p, &end, 10);
  if (end == p || *end != '.') return 0;
  *layer = static_cast<int>(l);
  *rest = std::string(end + 1);
  return 1;
}

// Where a logical tensor lives in the packed layout. grp/grp_stride/grp_off describe the
// row map (see rowops.cuh); f32 tensors (norms, biases) have dst_f32 set.
struct Slot {
  __nv_bfloat16* dst = nullptr;
  float* dst_f32 = nullptr;
  int64_t rows = 0, cols = 0;
  int64_t grp = 1, grp_stride = 1, grp_off = 0;
  int64_t f32_offset = 0;
  // the slot holds block [r0, r0 + rows) x [c0, c0 + cols) of a full_rows x full_cols logical tensor
  int64_t r0 = 0, c0 = 0, full_rows = 0, full_cols = 0;
};

int resolve_slot(drt_model* m, const char* key, Slot* out) {
  Slot s;
  const int64_t H = m->H;
  if (strcmp(key, "model.embed_tokens.weight") == 0) {
    s.dst = m->embed; s.rows = m->V; s.cols = H;
  } else if (strcmp(key, "lm_head.weight") == 0) {
    if (m->cfg.tied_lm_head) return set_error(DRT_INVALID_ARGUMENT, "lm_head.weight is tied to the embedding in this model");
    s.dst = m->lm_head; s.rows = m->V; s.cols = H;
  } else if (strcmp(key, "model.norm.weight") == 0) {
    s.dst_f32 = m->final_norm; s.rows = 1; s.cols = H;
  } else {
    int l = -1;
    std::string rest;
    if (!parse_layer_key(key, &l, &rest) || l < 0 || l >= m->L) return set_error(DRT_INVALID_ARGUMENT, "unknown weight key %s", key);
    LayerW& w = m->layers[l];
    const int64_t qr = static_cast<int64_t>(m->nq) * 128, kr = static_cast<int64_t>(m->nkv) * 128;
    const int64_t q0 = static_cast<int64_t>(m->shard.q_head0) * 128, k0 = static_cast<int64_t>(m->shard.kv_head0) * 128;
    const int64_t qf = static_cast<int64_t>(m->nq_full) * 128, kf = static_cast<int64_t>(m->nkv_full) * 128;
    if (rest == "self_attn.q_proj.weight") { s.r0 = q0; s.full_rows = qf; s.full_cols = H; }
    else if (rest == "self_attn.k_proj.weight" || rest == "self_attn.v_proj.weight") { s.r0 = k0; s.full_rows = kf; s.full_cols = H; }
    else if (rest == "self_attn.q_proj.bias") { s.c0 = q0; s.full_rows = 1; s.full_cols = qf; }
    else if (rest == "self_attn.k_proj.bias" || rest == "self_attn.v_proj.bias") { s.c0 = k0; s.full_rows = 1; s.full_cols = kf; }
    else if (rest == "self_attn.o_proj.weight") { s.c0 = q0; s.full_rows = H; s.full_cols = qf; }
    else if (rest == "mlp.gate_proj.weight" || rest == "mlp.up_proj.weight") { s.r0 = m->shard.inter0; s.full_rows = m->I_full; s.full_cols = H; }
    else if (rest == "mlp.down_proj.weight") { s.c0 = m->shard.inter0; s.full_rows = H; s.full_cols = m->I_full; }
    if (rest == "input_layernorm.weight") { s.dst_f32 = w.in_norm; s.rows = 1; s.cols = H; }
    else if (rest == "post_attention_layernorm.weight") { s.dst_f32 = w.post_norm; s.rows = 1; s.cols = H; }
    else if (rest == "self_attn.q_norm.weight") { if (!w.q_norm) return set_error(DRT_INVALID_ARGUMENT, "model has no QK norm"); s.dst_f32 = w.q_norm; s.rows = 1; s.cols = 128; }
    else if (rest == "self_attn.k_norm.weight") { if (!w.k_norm) return set_error(DRT_INVALID_ARGUMENT, "model has no QK norm"); s.dst_f32 = w.k_norm; s.rows = 1; s.cols = 128; }
    else if (rest == "self_attn.q_proj.weight") { s.dst = w.wqkv; s.rows = qr; s.cols = H; s.grp = qr; s.grp_stride = 0; s.grp_off = 0; }
    else if (rest == "self_attn.k_proj.weight") { s.dst = w.wqkv; s.rows = kr; s.cols = H; s.grp = kr; s.grp_stride = 0; s.grp_off = qr; }
    else if (rest == "self_attn.v_proj.weight") { s.dst = w.wqkv; s.rows = kr; s.cols = H; s.grp = kr; s.grp_stride = 0; s.grp_off = qr + kr; }
    else if (rest == "self_attn.q_proj.bias") { if (!w.bqkv) return set_error(DRT_INVALID_ARGUMENT, "model has no qkv bias"); s.dst_f32 = w.bqkv; s.rows = 1; s.cols = qr; s.f32_offset = 0; }
    else if (rest == "self_attn.k_proj.bias") { if (!w.bqkv) return set_error(DRT_INVALID_ARGUMENT, "model has no qkv bias"); s.dst_f32 = w.bqkv; s.rows = 1; s.cols = kr; s.f32_offset = qr; }
    else if (rest == "self_attn.v_proj.bias") { if (!w.bqkv) return set_error(DRT_INVALID_ARGUMENT, "model has no qkv bias"); s.dst_f32 = w.bqkv; s.rows = 1; s.cols = kr; s.f32_offset = qr + kr; }
    else if (rest == "self_attn.o_proj.weight") { s.dst = w.wo; s.rows = H; s.cols = qr; }
    else if (rest == "mlp.gate_proj.weight") { s.dst = w.wgu; s.rows = m->I; s.cols = H; s.grp = 64; s.grp_stride = 128; s.grp_off = 0; }
    else if (rest == "mlp.up_proj.weight") { s.dst = w.wgu; s.rows = m->I; s.cols = H; s.grp = 64; s.grp_stride = 128; s.grp_off = 64; }
    else if (rest == "mlp.down_proj.weight") { s.dst = w.wdown; s.rows = H; s.cols = m->I; }
    else return set_error(DRT_INVALID_ARGUMENT, "unknown weight key %s", key);
  }
  if (s.grp == 1 && s.grp_stride == 1) { s.grp = s.rows; s.grp_stride = 0; }
  if (s.full_rows == 0) { s.full_rows = s.rows; s.full_cols = s.cols; }
  *out = s;
  return DRT_OK;
}
}  // namespace

extern "C" int drt_abi_version(int32_t* major, int32_t* minor, int32_t* patch) {
  if (major) *major = DRT_ABI_VERSION_MAJOR;
  if (minor) *minor = DRT_ABI_VERSION_MINOR;
  if (patch) *patch = DRT_ABI_VERSION_PATCH;
  return DRT_OK;
}

extern "C" const char* drt_last_error(void) { return g_last_error.c_str(); }

extern "C" int drt_device_count(int32_t* count) {
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) n = 0;
  if (count) *count = n;
  return DRT_OK;
}

namespace {
int create_model(const drt_model_config* cfg, int32_t device, const drt_tp_shard* shard, drt_model** out);
}  // namespace

extern "C" int drt_model_create(const drt_model_config* cfg, int32_t device, drt_model** out) {
  REQUIRE(cfg != nullptr && out != nullptr, "null argument");
  *out = nullptr;
  drt_tp_shard whole;
  TRY(tp_geometry(cfg, 0, 1, &whole));
  return create_model(cfg, device, &whole, out);
}

extern "C" int drt_tp_shard_geometry(const drt_model_config* cfg, int32_t rank, int32_t world, drt_tp_shard* out) {
  REQUIRE(cfg != nullptr && out != nullptr, "null argument");
  return tp_geometry(cfg, rank, world, out);
}

extern "C" uint64_t drt_tp_flag_value(uint64_t epoch, int32_t layer, int32_t which) {
  return tp_flag_value(epoch, 2 * layer + which);
}

extern "C" int drt_tp_unique_id(uint8_t* id) {
  REQUIRE(id != nullptr, "null argument");
  const NcclApi* nc = nullptr;
  TRY(nccl_api(&nc));
  ncclUniqueId u;
  NCCL_CK(nc, nc->get_unique_id(&u));
  static_assert(sizeof(u.internal) == DRT_TP_ID_BYTES, "NCCL unique id size");
  memcpy(id, u.internal, DRT_TP_ID_BYTES);
  return DRT_OK;
}

extern "C" int drt_model_create_tp(const drt_model_config* cfg, int32_t device, int32_t rank, int32_t world,
                                   const uint8_t* nccl_id, drt_model** out) {
  REQUIRE(cfg != nullptr && out != nullptr && nccl_id != nullptr, "null argument");
  *out = nullptr;
  drt_tp_shard g;
  TRY(tp_geometry(cfg, rank, world, &g));
  const NcclApi* nc = nullptr;
  TRY(nccl_api(&nc));
  drt_model* m = nullptr;
  TRY(create_model(cfg, device, &g, &m));
  CK(cudaSetDevice(device));
  ncclUniqueId u;
  memcpy(u.internal, nccl_id, DRT_TP_ID_BYTES);
  ncclResult_t r = nc->comm_init_rank(&m->comm, world, u, rank);
  if (r != ncclSuccess) {
    m->comm = nullptr;
    drt_model_destroy(m);
    return set_error(DRT_INTERNAL_ERROR, "NCCL communicator: %s", nc->error_string(r));
  }
  *out = m;
  return DRT_OK;
}

namespace {
int create_model(const drt_model_config* cfg, int32_t device, const drt_tp_shard* shard, drt_model** out) {
  REQUIRE(cfg->head_dim == 128, "head_dim must be 128 (got %d)", cfg->head_dim);
  REQUIRE(cfg->layer_count > 0 && cfg->hidden_size > 0 && cfg->vocab_size > 0, "bad model geometry");
  REQUIRE(cfg->hidden_size % 128 == 0, "hidden_size must be a multiple of 128");
  REQUIRE(cfg->hidden_size <= 4 * kNormVec * 256, "hidden_size above %d", 4 * kNormVec * 256);
  REQUIRE(cfg->intermediate_size % 64 == 0, "intermediate_size must be a multiple of 64");
  REQUIRE(cfg->vocab_size % 128 == 0, "vocab_size must be a multiple of 128");
  REQUIRE(cfg->num_kv_heads > 0 && cfg->attention_heads % cfg->num_kv_heads == 0, "attention_heads must divide by num_kv_heads");
  REQUIRE(cfg->attention_heads / cfg->num_kv_heads <= 128, "GQA group too large");
  REQUIRE(cfg->max_seq > 0 && cfg->max_seq % 8 == 0, "max_seq must be a positive multiple of 8");
  CK(cudaSetDevice(device));
  TRY(configure_kernels());
  drt_model* m = new drt_model();
  m->cfg = *cfg;
  m->device = device;
  m->shard = *shard;
  m->nq_full = cfg->attention_heads;
  m->nkv_full = cfg->num_kv_heads;
  m->I_full = cfg->intermediate_size;
  m->H = cfg->hidden_size;
  m->nq = shard->q_heads;
  m->nkv = shard->kv_heads;
  m->I = shard->inter;
  m->V = cfg->vocab_size;
  m->L = cfg->layer_count;
  m->rep = m->nq / m->nkv;
  m->tile_pos = 128 / m->rep;
  m->qkv_rows = (m->nq + 2 * m->nkv) * 128;
  m->gu_rows = 2 * m->I;
  m->layers.resize(m->L);
  auto fail = [&](int rc) { drt_model_destroy(m); return rc; };
  int rc;
  if ((rc = dalloc(m, &m->embed, static_cast<size_t>(m->V) * m->H)) != DRT_OK) return fail(rc);
  if (cfg->tied_lm_head) m->lm_head = m->embed;
  else if ((rc = dalloc(m, &m->lm_head, static_cast<size_t>(m->V) * m->H)) != DRT_OK) return fail(rc);
  if ((rc = dalloc(m, &m->final_norm, m->H)) != DRT_OK) return fail(rc);
  for (int l = 0; l < m->L; ++l) {
    LayerW& w = m->layers[l];
    if ((rc = dalloc(m, &w.wqkv, static_cast<size_t>(m->qkv_rows) * m->H)) != DRT_OK) return fail(rc);
    if ((rc = dalloc(m, &w.wo, static_cast<size_t>(m->H) * m->nq * 128)) != DRT_OK) return fail(rc);
    if ((rc = dalloc(m, &w.wgu, static_cast<size_t>(m->gu_rows) * m->H)) != DRT_OK) return fail(rc);
    if ((rc = dalloc(m, &w.wdown, static_cast<size_t>(m->H) * m->I)) != DRT_OK) return fail(rc);
    if ((rc = dalloc(m, &w.in_norm, m->H)) != DRT_OK) return fail(rc);
    if ((rc = dalloc(m, &w.post_norm, m->H)) != DRT_OK) return fail(rc);
    if (cfg->qk_norm) {
      if ((rc = dalloc(m, &w.q_norm, 128)) != DRT_OK) return fail(rc);
      if ((rc = dalloc(m, &w.k_norm, 128)) != DRT_OK) return fail(rc);
    }
    if (cfg->qkv_bias && (rc = dalloc(m, &w.bqkv, m->qkv_rows)) != DRT_OK) return fail(rc);
    if ((rc = map_matrix(&w.m_qkv, w.wqkv, m->qkv_rows, m->H, 128)) != DRT_OK) return fail(rc);
    if ((rc = map_matrix(&w.m_o, w.wo, m->H, static_cast<int64_t>(m->nq) * 128, 128)) != DRT_OK) return fail(rc);
    if ((rc = map_matrix(&w.m_gu, w.wgu, m->gu_rows, m->H, 128)) != DRT_OK) return fail(rc);
    if ((rc = map_matrix(&w.m_down, w.wdown, m->H, m->I, 128)) != DRT_OK) return fail(rc);
  }
  if ((rc = map_matrix(&m->m_lm, m->lm_head, m->V, m->H, 128)) != DRT_OK) return fail(rc);
  // Norm weights default to 1; RoPE tables default to the host float32 construction.
  if ((rc = fill_f32(m->final_norm, m->H, 1.0f, 0)) != DRT_OK) return fail(rc);
  for (auto& w : m->layers) {
    if ((rc = fill_f32(w.in_norm, m->H, 1.0f, 0)) != DRT_OK) return fail(rc);
    if ((rc = fill_f32(w.post_norm, m->H, 1.0f, 0)) != DRT_OK) return fail(rc);
    if (w.q_norm && (rc = fill_f32(w.q_norm, 128, 1.0f, 0)) != DRT_OK) return fail(rc);
    if (w.k_norm && (rc = fill_f32(w.k_norm, 128, 1.0f, 0)) != DRT_OK) return fail(rc);
    if (w.bqkv && (rc = fill_f32(w.bqkv, m->qkv_rows, 0.0f, 0)) != DRT_OK) return fail(rc);
  }
  {
    std::vector<float> c, s;
    host_rope(c, s, cfg->max_seq, cfg->rope_theta);
    if ((rc = drt_model_set_rope(m, c.data(), s.data(), cfg->max_seq)) != DRT_OK) return fail(rc);
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(set_error(DRT_INTERNAL_ERROR, "model init failed: %s", cudaGetErrorString(cudaGetLastError())));
  *out = m;
  return DRT_OK;
}
}  // namespace

extern "C" int drt_model_set_rope(drt_model* m, const float* cos_half, const float* sin_half, int32_t n_pos) {
  REQUIRE(m && cos_half && sin_half && n_pos > 0, "null argument");
  CK(cudaSetDevice(m->device));
  if (m->rope_pos < n_pos) {
    int rc;
    if ((rc = dalloc(m, &m->rope_cos, static_cast<size_t>(n_pos) * 64)) != DRT_OK) return rc;
    if ((rc = dalloc(m, &m->rope_sin, static_cast<size_t>(n_pos) * 64)) != DRT_OK) return rc;
  }
  CK(cudaMemcpy(m->rope_cos, cos_half, sizeof(float) * n_pos * 64, cudaMemcpyHostToDevice));
  CK(cudaMemcpy(m->rope_sin, sin_half, sizeof(float) * n_pos * 64, cudaMemcpyHostToDevice));
  m->rope_pos = n_pos;
  return DRT_OK;
}

extern "C" int drt_model_init_synthetic(drt_model* m, uint64_t seed, float linear_std, float embed_std, float bias_std) {
  REQUIRE(m != nullptr, "null model");
  CK(cudaSetDevice(m->device));
  const double unit = std::sqrt(21845.0);  // std of the 4-byte Irwin-Hall sum
  const float s_lin = static_cast<float>(static_cast<double>(linear_std) / unit);
  const float s_emb = static_cast<float>(static_cast<double>(embed_std) / unit);
  const float s_bias = static_cast<float>(static_cast<double>(bias_std) / unit);
  // (r0, c0, full_cols): the block of the logical tensor this model holds (tensor-parallel shards)
  auto fill = [&](__nv_bfloat16* dst, int64_t rows, int64_t cols, uint32_t tid, float scale, int64_t grp, int64_t grp_stride,
                  int64_t grp_off, int64_t r0 = 0, int64_t c0 = 0, int64_t full_cols = 0) -> int {
    const int64_t total = rows * cols;
    const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 65535));
    synth_fill_kernel<<<blocks, 256>>>(dst, rows, cols, seed, tid, scale, grp, grp_stride, grp_off, r0, c0,
                                       full_cols > 0 ? full_cols : cols);
    CK(cudaGetLastError());
    return DRT_OK;
  };
  const int64_t H = m->H, qr = static_cast<int64_t>(m->nq) * 128, kr = static_cast<int64_t>(m->nkv) * 128;
  const int64_t q0 = static_cast<int64_t>(m->shard.q_head0) * 128, k0 = static_cast<int64_t>(m->shard.kv_head0) * 128;
  const int64_t qf = static_cast<int64_t>(m->nq_full) * 128, kf = static_cast<int64_t>(m->nkv_full) * 128;
  const int64_t i0 = m->shard.inter0;
  TRY(fill(m->embed, m->V, H, 1, s_emb, m->V, 0, 0));
  if (!m->cfg.tied_lm_head) TRY(fill(m->lm_head, m->V, H, 2, s_emb, m->V, 0, 0));
  for (int l = 0; l < m->L; ++l) {
    LayerW& w = m->layers[l];
    const uint32_t b = 16u + static_cast<uint32_t>(l) * 16u;
    TRY(fill(w.wqkv, qr, H, b + 0, s_lin, qr, 0, 0, q0, 0, H));
    TRY(fill(w.wqkv, kr, H, b + 1, s_lin, kr, 0, qr, k0, 0, H));
    TRY(fill(w.wqkv, kr, H, b + 2, s_lin, kr, 0, qr + kr, k0, 0, H));
    TRY(fill(w.wo, H, qr, b + 3, s_lin, H, 0, 0, 0, q0, qf));
    TRY(fill(w.wgu, m->I, H, b + 4, s_lin, 64, 128, 0, i0, 0, H));
    TRY(fill(w.wgu, m->I, H, b + 5, s_lin, 64, 128, 64, i0, 0, H));
    TRY(fill(w.wdown, H, m->I, b + 6, s_lin, H, 0, 0, 0, i0, m->I_full));
    if (w.bqkv) {
      // Biases are bf16 values held in f32: generate bf16 into a scratch row, widen.
      __nv_bfloat16* tmp = nullptr;
      CK(cudaMalloc(&tmp, sizeof(__nv_bfloat16) * m->qkv_rows));
      int rc = fill(tmp, 1, qr, b + 7, s_bias, 1, 0, 0, 0, q0, qf);
      if (rc == DRT_OK) rc = fill(tmp + qr, 1, kr, b + 8, s_bias, 1, 0, 0, 0, k0, kf);
      if (rc == DRT_OK) rc = fill(tmp + qr + kr, 1, kr, b + 9, s_bias, 1, 0, 0, 0, k0, kf);
      if (rc == DRT_OK) {
        bf16_to_f32_kernel<<<64, 256>>>(w.bqkv, tmp, m->qkv_rows);
        if (cudaGetLastError() != cudaSuccess) rc = set_error(DRT_INTERNAL_ERROR, "bias widen failed");
      }
      cudaDeviceSynchronize();
      cudaFree(tmp);
      TRY(rc);
    }
  }
  CK(cudaDeviceSynchronize());
  return DRT_OK;
}

extern "C" int drt_model_set_tensor(drt_model* m, const char* key, const void* data, int32_t dtype, int64_t rows, int64_t cols) {
  REQUIRE(m && key && data, "null argument");
  REQUIRE(dtype == 0 || dtype == 1, "dtype must be 0 (bf16) or 1 (f32)");
  Slot s;
  TRY(resolve_slot(m, key, &s));
  REQUIRE(rows * cols == s.full_rows * s.full_cols, "%s: expected %lld x %lld elements, got %lld x %lld", key,
          static_cast<long long>(s.full_rows), static_cast<long long>(s.full_cols), static_cast<long long>(rows),
          static_cast<long long>(cols));
  CK(cudaSetDevice(m->device));
  const int64_t n = s.rows * s.cols;
  // A tensor-parallel shard takes its block of the full logical tensor.
  std::vector<uint8_t> block;
  if (s.rows != s.full_rows || s.cols != s.full_cols) {
    const size_t es = dtype == 1 ? 4 : 2;
    block.resize(static_cast<size_t>(n) * es);
    for (int64_t r = 0; r < s.rows; ++r)
      memcpy(block.data() + static_cast<size_t>(r * s.cols) * es,
             static_cast<const uint8_t*>(data) + static_cast<size_t>((s.r0 + r) * s.full_cols + s.c0) * es,
             static_cast<size_t>(s.cols) * es);
    data = block.data();
  }
  if (s.dst_f32 != nullptr) {
    std::vector<float> tmp(n);
    if (dtype == 1) {
      memcpy(tmp.data(), data, sizeof(float) * n);
    } else {
      const uint16_t* src = static_cast<const uint16_t*>(data);
      for (int64_t i = 0; i < n; ++i) {
        uint32_t bits = static_cast<uint32_t>(src[i]) << 16;
        memcpy(&tmp[i], &bits, 4);
      }
    }
    CK(cudaMemcpy(s.dst_f32 + s.f32_offset, tmp.data(), sizeof(float) * n, cudaMemcpyHostToDevice));
    return DRT_OK;
  }
  REQUIRE(dtype == 0, "%s: matrices must be bf16", key);
  __nv_bfloat16* staging = nullptr;
  CK(cudaMalloc(&staging, sizeof(__nv_bfloat16) * n));
  cudaError_t e = cudaMemcpy(staging, data, sizeof(__nv_bfloat16) * n, cudaMemcpyHostToDevice);
  if (e == cudaSuccess) {
    const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 65535));
    pack_rows_kernel<<<blocks, 256>>>(s.dst, staging, s.rows, s.cols, s.grp, s.grp_stride, s.grp_off);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
  }
  cudaFree(staging);
  if (e != cudaSuccess) return set_error(DRT_INTERNAL_ERROR, "set_tensor %s: %s", key, cudaGetErrorString(e));
  return DRT_OK;
}

extern "C" int drt_model_get_tensor(drt_model* m, const char* key, void* data, int32_t dtype, int64_t rows, int64_t cols) {
  REQUIRE(m && key && data, "null argument");
  REQUIRE(dtype == 0 || dtype == 1, "dtype must be 0 (bf16) or 1 (f32)");
  Slot s;
  TRY(resolve_slot(m, key, &s));
  REQUIRE(rows * cols == s.rows * s.cols, "%s: element count mismatch (a tensor-parallel shard returns its own block)", key);
  CK(cudaSetDevice(m->device));
  const int64_t n = s.rows * s.cols;
  if (s.dst_f32 != nullptr) {
    std::vector<float> tmp(n);
    CK(cudaMemcpy(tmp.data(), s.dst_f32 + s.f32_offset, sizeof(float) * n, cudaMemcpyDeviceToHost));
    if (dtype == 1) {
      memcpy(data, tmp.data(), sizeof(float) * n);
    } else {
      uint16_t* dst = static_cast<uint16_t*>(data);
      for (int64_t i = 0; i < n; ++i) {
        uint32_t bits;
        memcpy(&bits, &tmp[i], 4);
        dst[i] = static_cast<uint16_t>(bits >> 16);
      }
    }
    return DRT_OK;
  }
  std::vector<uint16_t> row(static_cast<size_t>(s.cols));
  for (int64_t r = 0; r < s.rows; ++r) {
    const int64_t dr = (r / s.grp) * s.grp_stride + s.grp_off + r % s.grp;
    CK(cudaMemcpy(row.data(), s.dst + dr * s.cols, sizeof(uint16_t) * s.cols, cudaMemcpyDeviceToHost));
    if (dtype == 0) {
      memcpy(static_cast<uint16_t*>(data) + r * s.cols, row.data(), sizeof(uint16_t) * s.cols);
    } else {
      float* dst = static_cast<float*>(data) + r * s.cols;
      for (int64_t c = 0; c < s.cols; ++c) {
        uint32_t bits = static_cast<uint32_t>(row[c]) << 16;
        memcpy(&dst[c], &bits, 4);
      }
    }
  }
  return DRT_OK;
}

namespace {
// (Re)build the 4-bit copy of the bf16 weight w [n][K].
int quantize_into(drt_model* m, QuantW* qw, const __nv_bfloat16* w, int64_t n, int64_t K, int bits) {
  if (qw->bits_cap < bits) {  // a narrower earlier buffer stays with the model's allocations
    TRY(dalloc(m, &qw->q, static_cast<size_t>(n) * K * bits / 8));
    qw->bits_cap = bits;
  }
  if (qw->scale == nullptr) {
    TRY(dalloc(m, &qw->scale, static_cast<size_t>(n) * (K / 64)));
    TRY(dalloc(m, &qw->bias, static_cast<size_t>(n) * (K / 64)));
  }
  TRY(map_u8(&qw->map, qw->q, n, K * bits / 8, 64 * bits / 8, 128));
  const int64_t total = n * (K / 64);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 65535));
  if (bits == 8)
    quantize_q8_kernel<<<blocks, 256>>>(w, n, static_cast<int>(K), qw->q, qw->scale, qw->bias);
  else
    quantize_q4_kernel<<<blocks, 256>>>(w, n, static_cast<int>(K), qw->q, qw->scale, qw->bias);
  CK(cudaGetLastError());
  return DRT_OK;
}
}  // namespace

extern "C" int drt_model_quantize(drt_model* m, int32_t bits, int32_t group_size) {
  REQUIRE(m, "null model");
  REQUIRE(m->shard.world == 1, "4-bit linears are served on whole (not tensor-parallel) models");
  if ((bits != 4 && bits != 8) || group_size != 64)
    return set_error(DRT_UNSUPPORTED, "linear quantization serves bits 4 or 8 with group size 64 (got bits %d, group %d)",
                     bits, group_size);
  REQUIRE(m->H % 64 == 0 && m->I % 64 == 0, "linear in-dims must be multiples of the group size");
  CK(cudaSetDevice(m->device));
  const int64_t H = m->H, I = m->I, qd = static_cast<int64_t>(m->nq) * 128;
  for (int l = 0; l < m->L; ++l) {
    LayerW& w = m->layers[l];
    TRY(quantize_into(m, &w.q_qkv, w.wqkv, m->qkv_rows, H, bits));
    TRY(quantize_into(m, &w.q_o, w.wo, H, qd, bits));
    TRY(quantize_into(m, &w.q_gu, w.wgu, m->gu_rows, H, bits));
    TRY(quantize_into(m, &w.q_down, w.wdown, H, I, bits));
  }
  TRY(quantize_into(m, &m->q_lm, m->lm_head, m->V, H, bits));
  CK(cudaDeviceSynchronize());
  m->quantized = true;
  m->qbits = bits;
  return DRT_OK;
}

extern "C" int64_t drt_model_device_bytes(const drt_model* m) { return m ? m->bytes : 0; }

extern "C" void drt_model_destroy(drt_model* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  cudaDeviceSynchronize();
  if (m->comm != nullptr) {
    const NcclApi* nc = nullptr;
    if (nccl_api(&nc) == DRT_OK) nc->comm_destroy(m->comm);
    m->comm = nullptr;
  }
  for (void* p : m->allocs) cudaFree(p);
  delete m;
}

// ======================================================================= session
struct drt_session {
  drt_model* m = nullptr;
  drt_session_config cfg;
  int device = 0;
  int max_seq = 0, rows_cap = 0, planes = 0;
  std::vector<void*> allocs;
  int64_t bytes = 0;
  cudaStream_t stream = nullptr;
  // device buffers
  int* canvas = nullptr;
  float* h = nullptr;
  __nv_bfloat16 *xn = nullptr, *q = nullptr, *attn = nullptr, *act = nullptr, *xf = nullptr;
  float* logits = nullptr;
  float* part = nullptr;              // [rows_cap][H] f32 linear partials (tensor-parallel models)
  // tensor parallel over peer memory: receive buffers [2][world][rows_cap][H] f32, all-gather
  // buffers [2][rows_cap][H] bf16, flags [3][2][kTpMaxRanks] u64 and the logits [head_cap][V] f32,
  // in one allocation shared with the peers through CUDA IPC
  uint8_t* tp_buf = nullptr;
  uint8_t* tp_peer[kTpMaxRanks] = {};
  bool tp_p2p = false;
  // vocabulary-parallel lm_head (peers mapped): this rank projects vocabulary tiles
  // [lm_t0, lm_t0 + lm_tiles) and stores them into every rank's logits
  bool tp_vocab = false;
  int lm_t0 = 0, lm_tiles = 0;
  CUtensorMap m_lm_shard;
  int* tp_count = nullptr;            // [5] arrival counters: pushing linears [2], reduce-scatter [2], lm_head gather
  unsigned long long* tp_epoch = nullptr;
  __nv_bfloat16 *kcache = nullptr, *vtcache = nullptr;
  int max_cluster = 16;               // largest cluster the GPU schedules for the split kernels
  float* sel_pmax = nullptr;
  int* sel_pidx = nullptr;
  double* sel_psum = nullptr;
  int* sel_cnt = nullptr;
  double *sel_skey = nullptr, *sel_skey2 = nullptr;  // sampled-key chunk partials (temperature > 0)
  int* sel_sidx = nullptr;
  double *sel_amax = nullptr, *sel_sum = nullptr, *conf = nullptr;
  int* token = nullptr;
  int* scope_rows = nullptr;
  int* status = nullptr;
  DecodeState* state = nullptr;
  StepTrace* trace = nullptr;
  int trace_cap = 0;
  // host mirrors
  DecodeState* hstate = nullptr;   // pinned
  int* hflags = nullptr;           // pinned ring of stopped flags
  int canvas_len = 0;
  int origin = 0, block_size = 32, mask_id = 0;
  bool started = false;
  bool exact_kv = true;               // propose reuses the frozen prefix's K/V (false: recompute it)
  int propose_count = 0;              // forwards since start_device (keys the sampled draws)
  // launch geometry
  int sms = 148;
  int attn_splits = 1, attn_tps = 1;
  int sel_chunks = 1;
  // tensor maps over the activation buffers
  CUtensorMap m_xn64, m_xn128, m_xn256, m_attn64, m_attn128, m_attn256, m_act64, m_act128, m_act256, m_xf64, m_q, m_k, m_v;
  CUtensorMap m_k64;                  // K cache with 64-key boxes (decode attention)
  float* sk_part = nullptr;           // stream-K linears: per-CTA partial tiles [SMs][128][128] f32
  int* sk_flag = nullptr;             // and their ready flags [SMs] (zero between launches)
  int da_splits = 0;                  // decode attention CTAs per KV head (0: use attn_prefix_kernel)
  int da_cluster = 0;                 // the splits of a KV head run as one cluster and merge in it
  float* da_part_o = nullptr;         // decode attention split partials
  float* da_part_ml = nullptr;
  // graphs
  int g_step_kernels = 0;             // kernels in one replay of g_step
  cudaGraphExec_t g_step = nullptr;   // plan + forward + score + commit
  cudaGraphExec_t g_fwd = nullptr;    // forward + score (host policy)
  int g_step_geom[3] = {-1, -1, -1};  // (mask origin, block size, sampling selector) baked into each graph
  int g_fwd_geom[3] = {-1, -1, -1};
  int cap_sample = 0;                 // the graph being captured draws sampled tokens (temperature > 0)
  cudaEvent_t ev0 = nullptr, ev1 = nullptr;
  // full-canvas (entropy_count) sessions
  bool dream = false;
  int head_cap = kMaxFrontier;        // rows the final-norm / lm_head / selector buffers hold
  int* row_tie = nullptr;             // [head_cap] per-row certification bits (top-p selector)
  DreamState* dstate = nullptr;
  DreamState* hdstate = nullptr;      // pinned
  int* d_fpos = nullptr;              // [head_cap] frontier positions
  int* d_klist = nullptr;             // transfer count per proceeding step
  int* d_stepof = nullptr;            // loop step of each proceeding step
  int d_steps_cap = 0;
  CUtensorMap m_xf128, m_xf256;
  cudaGraphExec_t g_dream = nullptr;  // plan + full-canvas forward + head + top-p score + commit
  int g_dream_kernels = 0;
  struct DreamKey {
    int canvas_len, prompt_len, mask_id;
    double temperature, top_p;
    StepTrace* trace;
  } g_dream_key = {-1, -1, -1, 0.0, 0.0, nullptr};
  // metrics
  int64_t m_forwards = 0, m_rows = 0, m_prefill_rows = 0, m_committed = 0, m_near = 0, m_exact = 0;
  double m_ms = 0.0;
};

namespace {
template <typename T>
int salloc(drt_session* s, T** p, size_t count) {
  void* q = nullptr;
  CK(cudaMalloc(&q, std::max<size_t>(count * sizeof(T), 256)));
  s->allocs.push_back(q);
  s->bytes += static_cast<int64_t>(count * sizeof(T));
  *p = static_cast<T*>(q);
  return DRT_OK;
}

// One rank's tensor-parallel buffer: receive [2][world][slot] f32 partials, all-gather [2][slot]
// bf16 sums, reduce-scatter flags [2][kTpMaxRanks] and all-gather flags [2][kTpMaxRanks] (u64).
size_t tp_buf_bytes(const drt_session* s) {
  const size_t slot = static_cast<size_t>(s->rows_cap) * s->m->H;
  const size_t flags = 6 * kTpMaxRanks * sizeof(unsigned long long);
  const size_t head = (2 * static_cast<size_t>(s->m->shard.world) * slot * sizeof(float) + 2 * slot * sizeof(__nv_bfloat16) +
                       flags + 255) / 256 * 256;
  return head + static_cast<size_t>(s->head_cap) * s->m->V * sizeof(float);
}

int check_status(drt_session* s) {
  int code = 0;
  CK(cudaMemcpy(&code, s->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (code != 0) {
    cudaMemset(s->status, 0, sizeof(int));
    // a wait that ran out may have left stream-K ready flags raised
    if (s->sk_flag != nullptr) cudaMemset(s->sk_flag, 0, sizeof(int) * s->sms);
    if (code == DEV_BAD_SHAPE) return set_error(DRT_INVALID_ARGUMENT, "device rejected an input (token id out of range)");
    if (code == DEV_TIMEOUT_PEER) return set_error(DRT_DEVICE_TIMEOUT, "a tensor-parallel peer did not deliver its partials in time");
    if (code == DEV_BAD_GEOMETRY) return set_error(DRT_INTERNAL_ERROR, "a kernel's launch geometry did not cover its work");
    return set_error(DRT_DEVICE_TIMEOUT, "device wait expired (code %d)", code);
  }
  return DRT_OK;
}

struct Fwd {
  bool decode;                 // static decode shapes (graph-capturable)
  int rows;                    // rows covered by the grid
  const int* rows_dev;
  int pos0;
  const int* pos0_dev;
  int kv_len;
  const int* kv_len_dev;
  int prompt_len, block_size, bidirectional;
};

GemmArgs base_args(drt_session* s, int n_out, int K, const Fwd& f) {
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.n_out = n_out;
  a.K = K;
  a.rows = f.rows;
  a.rows_dev = f.rows_dev;
  a.splits = 1;
  a.kb_per_split = K / 64;
  a.status = s->status;
  a.pos0 = f.pos0;
  a.pos0_dev = f.pos0_dev;
  return a;
}

constexpr size_t kHalfSmPrefill = 113 * 1024;   // two CTAs share an SM
constexpr size_t kFullSmPrefill = 227 * 1024;   // one CTA per SM

template <int BN, int KS>
int launch_wide(drt_session* s, const CUtensorMap& mA, const CUtensorMap& mB, GemmArgs a, size_t smem_cap) {
  using Cfg = GemmCfg<BN, KS>;
  const int tiles_m = a.n_out / 128;
  const int tiles_n = (a.rows + BN - 1) / BN;
  a.splits = 1;
  a.kb_per_split = a.K / 64;
  int stages = 1;
  while (Cfg::smem_bytes(stages + 1) <= smem_cap) ++stages;
  a.stages = std::max(1, std::min((a.kb_per_split + KS - 1) / KS, stages));
  CK(launch_kc(gemm_swapab_kernel<BN, KS>, dim3(tiles_m, tiles_n, 1), dim3(128), Cfg::smem_bytes(a.stages), s->stream,
               true, 1, mA, mB, a));
  return DRT_OK;
}

// Linear over a wide activation block (prompt prefill, full-canvas forward, wide lm_head). Tile and
// ring shape from the measured B200 behaviour: one CTA's TMA ingest is bound by bytes per barrier
// round trip, so
//   * with at least two CTAs per SM of 256-row tiles: 128 x 256 tiles, two CTAs per SM (one CTA's
//     epilogue overlaps the other's main loop);
//   * with at most one wave of 128 x 128 tiles: one CTA per SM, two K blocks per stage, three stages;
//   * otherwise: 128 x 128 tiles, two CTAs per SM.
// mB128 / mB256: the activation map with 128- / 256-row boxes (mB256 null when the buffer is
// narrower than 256 rows).
// Stream-K linear (gemm_streamk_kernel): one CTA per SM takes an equal share of the (tile, K block)
// iterations. BN: activation rows per tile (mB's box).
template <int BN>
int launch_streamk(drt_session* s, const CUtensorMap& mA, const CUtensorMap& mB, GemmArgs a) {
  using Cfg = GemmCfg<BN, 2>;
  const long long total = static_cast<long long>(a.n_out / 128) * ((a.rows + BN - 1) / BN) * (a.K / 64);
  const int grid = static_cast<int>(std::min<long long>(s->sms, total));
  a.splits = 1;
  a.kb_per_split = a.K / 64;
  int stages = 1;
  while (Cfg::smem_bytes(stages + 1) <= kFullSmPrefill) ++stages;
  a.stages = stages;
  a.sk_part = s->sk_part;
  a.sk_flag = s->sk_flag;
  CK(launch_k(gemm_streamk_kernel<BN, 2>, dim3(grid), dim3(128), Cfg::smem_bytes(a.stages), s->stream, true, mA, mB, a));
  return DRT_OK;
}

int run_wide(drt_session* s, const CUtensorMap& mA, const CUtensorMap& mB128, const CUtensorMap* mB256, GemmArgs a) {
  const int tiles_m = a.n_out / 128;
  const int t256 = tiles_m * ((a.rows + 255) / 256);
  const int t128 = tiles_m * ((a.rows + 127) / 128);
  // One row tile (a decode window) on fewer weight tiles than nine tenths of the SMs, with K long
  // enough for many K blocks per CTA: the linear is a weight stream that one CTA per tile would read
  // on a fraction of the SMs. (Full-canvas shapes stay one CTA per tile: with several row tiles the
  // linear is compute-bound under the power cap, where waking the idle SMs measured slower.)
  const bool sk_epi = a.epi == EPI_RESID || a.epi == EPI_STORE_F32 || a.epi == EPI_STORE_RAW;
  if (s->sk_part != nullptr && sk_epi && a.rows <= 128 && t128 * 10 < s->sms * 9 &&
      t128 * (a.K / 64) >= 16 * s->sms)
    return launch_streamk<128>(s, mA, mB128, a);
  if (mB256 != nullptr && a.rows > 128 && t256 >= 2 * s->sms) return launch_wide<256, 1>(s, mA, *mB256, a, kHalfSmPrefill);
  if (t128 <= s->sms) return launch_wide<128, 2>(s, mA, mB128, a, kFullSmPrefill);
  return launch_wide<128, 1>(s, mA, mB128, a, kHalfSmPrefill);
}

// Split-K factor for the decode linears: the fewest K blocks per CTA with at most one CTA per SM,
// and the smallest factor among those that tie.
void dec_split(int tiles, int kb, int sms, int max_split, int* splits, int* kbps) {
  int best = 1, best_kb = kb;
  for (int sp = 2; sp <= std::min(max_split, kb); ++sp) {
    if (tiles * sp > sms) break;
    if (!dec_split_supported(sp)) continue;
    const int k = (kb + sp - 1) / sp;
    if (k < best_kb) {
      best = sp;
      best_kb = k;
    }
  }
  *splits = best;
  *kbps = best_kb;
}

// Decode linear over at most kDecRows activation rows (mB: the bf16 activation map, box 64 rows);
// q: the weight's 4-bit copy when the model is quantized (tmA then maps the packed nibbles).
// mB128: the same activation with 128-row boxes, for K too long for the decode kernel's resident
// activation slice even at the largest split (the wide linear then takes the shape).
int run_dec_gemm(drt_session* s, const CUtensorMap& mA, const CUtensorMap& mB, GemmArgs a, const QuantW* q = nullptr,
                 const CUtensorMap* mB128 = nullptr) {
  const int tiles_m = a.n_out / 128;
  const int kb = a.K / 64;
  if (q == nullptr && a.epi == EPI_STORE_F32 && tiles_m >= 2 * s->sms && kb <= kLmMaxKb) {
    // Vocabulary projection: one persistent CTA per SM over a contiguous run of weight tiles, the
    // deepest weight ring that fits beside the resident activation tile.
    const size_t budget = 227 * 1024;
    int stages = 0;
    while (stages < 8 && lm_smem_bytes(stages + 1, kb) <= budget) ++stages;
    if (stages < 2) return set_error(DRT_INTERNAL_ERROR, "lm_head ring does not fit (K = %d)", a.K);
    a.stages = stages;
    a.splits = 1;
    a.kb_per_split = kb;
    CK(launch_k(gemm_lm_kernel, dim3(std::min(tiles_m, s->sms)), dim3(kLmThreads), lm_smem_bytes(stages, kb), s->stream,
                true, mA, mB, a));
    return DRT_OK;
  }
  // Large bf16 weights (a 7B model's MLP and vocabulary projection) over a decode window: the
  // linear is a weight stream; stream-K over every SM reads it at a higher rate than one split-K
  // cluster per weight tile (Dream-7B D2F decode step: 6.67 -> 5.31 ms with the down_proj alone).
  if (q == nullptr && s->sk_part != nullptr && a.rows <= 64 &&
      static_cast<size_t>(a.n_out) * a.K * 2 >= (size_t{64} << 20) &&
      (a.epi == EPI_RESID || a.epi == EPI_STORE_F32 || a.epi == EPI_STORE_RAW || a.epi == EPI_SWIGLU))
    return launch_streamk<64>(s, mA, mB, a);
  dec_split(tiles_m, kb, s->sms, s->max_cluster, &a.splits, &a.kb_per_split);
  if (q != nullptr) {
    // every packed tile of a CTA's K slice stays resident: at most kDecQMaxKb blocks per CTA
    while (a.kb_per_split > kDecQMaxKb && a.splits < std::min(16, s->max_cluster)) {
      a.splits *= 2;
      a.kb_per_split = (kb + a.splits - 1) / a.splits;
    }
    if (a.kb_per_split > kDecQMaxKb) return set_error(DRT_UNSUPPORTED, "quantized linear with %d K blocks per CTA", a.kb_per_split);
    a.q_scale = q->scale;
    a.q_bias = q->bias;
    a.q_groups = kb;
    a.stages = kDecQStages;
    DecGemmKernel kern = dec_gemm_kernel(a.epi, a.splits, s->m->qbits);
    if (kern == nullptr) return set_error(DRT_INTERNAL_ERROR, "no quantized decode linear for epilogue %d, split %d", a.epi, a.splits);
    CK(launch_kc(kern, dim3(tiles_m, 1, a.splits), dim3(128), dec_q_smem_bytes(a.kb_per_split, s->m->qbits), s->stream, true, a.splits,
                 q->map, mB, a));
    return DRT_OK;
  }
  if (a.kb_per_split > kDecMaxKb) {
    // Long K (Dream-7B's MLP): more split-K CTAs than one per SM, in several waves, so that each
    // CTA's activation slice stays resident; beyond the largest cluster, the wide linear.
    int sp = a.splits;
    while (sp < std::min(16, s->max_cluster) && (kb + sp - 1) / sp > kDecMaxKb) sp *= 2;
    if ((kb + sp - 1) / sp <= kDecMaxKb) {
      a.splits = sp;
      a.kb_per_split = (kb + sp - 1) / sp;
    } else if (mB128 != nullptr) {
      return run_wide(s, mA, *mB128, nullptr, a);
    } else {
      return set_error(DRT_UNSUPPORTED, "decode linear with %d K blocks per CTA", a.kb_per_split);
    }
  }
  // Ring depth: the deepest ring (up to the whole K slice) that still lets two CTAs share an SM,
  // so the next kernel's CTAs can stream their weights beside this one; when that leaves fewer
  // than four stages for a longer slice, the whole slice in one CTA per SM instead.
  constexpr size_t kHalfSm = 115712;  // (228 KB - 2 x 1 KB reserved) / 2
  constexpr size_t kFullSm = 218 * 1024;
  int s_co = 0, s_full = 1;
  for (int st = 1; st <= a.kb_per_split; ++st) {
    if (dec_smem_bytes(st, a.kb_per_split) <= kHalfSm) s_co = st;
    if (dec_smem_bytes(st, a.kb_per_split) <= kFullSm) s_full = st;
  }
  a.stages = (s_co >= std::min(a.kb_per_split, 4)) ? s_co : s_full;
  DecGemmKernel kern = dec_gemm_kernel(a.epi, a.splits);
  if (kern == nullptr) return set_error(DRT_INTERNAL_ERROR, "no decode linear for epilogue %d, split %d", a.epi, a.splits);
  CK(launch_kc(kern, dim3(tiles_m, 1, a.splits), dim3(128), dec_smem_bytes(a.stages, a.kb_per_split), s->stream, true,
               a.splits, mA, mB, a));
  return DRT_OK;
}

int run_rmsnorm(drt_session* s, const float* h, const int* row_index, int rows, const int* rows_dev, const float* w,
                __nv_bfloat16* out) {
  drt_model* m = s->m;
  CK(launch_k(rmsnorm_bf16_kernel, dim3(rows), dim3(256), 0, s->stream, true, h, m->H, row_index, rows, rows_dev, w,
              m->cfg.rms_norm_eps, m->H, out, m->H));
  return DRT_OK;
}

// Peer-memory layout of one rank's tensor-parallel buffer (see tp_buf_bytes).
size_t tp_slot(const drt_session* s) { return static_cast<size_t>(s->rows_cap) * s->m->H; }
size_t tp_recv_offset(const drt_session* s, int b, int src) {
  return (static_cast<size_t>(b) * s->m->shard.world + src) * tp_slot(s) * sizeof(float);
}
size_t tp_ag_offset(const drt_session* s, int b) {
  return tp_recv_offset(s, 2, 0) + static_cast<size_t>(b) * tp_slot(s) * sizeof(__nv_bfloat16);
}
size_t tp_flag_offset(const drt_session* s, int kind, int b, int src) {  // kind 0: reduce-scatter, 1: all-gather, 2: lm_head
  return tp_ag_offset(s, 2) + ((static_cast<size_t>(kind) * 2 + b) * kTpMaxRanks + src) * sizeof(unsigned long long);
}
size_t tp_logits_offset(const drt_session* s) { return (tp_flag_offset(s, 3, 0, 0) + 255) / 256 * 256; }

// Tensor parallel over peer memory, for one row-split linear (o_proj: buffer 0, down_proj: 1):
//   1. the linear (EPI_TP_PUSH) stores each f32 partial tile into this rank's slot of the receive
//      buffer of the rank owning the tile's features and, when all its tiles are out, raises this
//      rank's reduce-scatter flag on every rank;
//   2. tp_rs_kernel: once every rank's partials are in, the owner sums them (rank order), adds
//      bf16(sum) to its residual and stores bf16(sum) into the other ranks' all-gather buffers, then
//      raises its all-gather flag on every rank;
//   3. tp_ag_kernel: once every owner's sums are in, each rank adds the sums of the tiles it does
//      not own.
// Every rank adds the same bf16 values, so the residuals stay bit-identical. A rank writes a
// buffer again only after it has seen every peer's flag of a later stage that follows the peer's
// last read of it (stream order on the peer), so two alternating buffers suffice.
// With two ranks the exchange is one step instead: each linear stores its whole partial into both
// ranks' buffers and tp_reduce_all_kernel sums them (the same bytes cross NVLink, with one kernel
// and one flag round trip fewer; measured 7.9 against 8.5 ms per Dream step).
int tp_push_linear(drt_session* s, const CUtensorMap& mA, const CUtensorMap& mB128, const CUtensorMap* mB256, GemmArgs a,
                   int b, int tag, int rows) {
  drt_model* m = s->m;
  const int world = m->shard.world, me = m->shard.rank;
  a.epi = EPI_TP_PUSH;
  a.ld_out = m->H;
  a.tp_world = world;
  a.tp_tag = tag;
  a.tp_count = s->tp_count + b;
  a.tp_epoch = s->tp_epoch;
  a.tp_all = world == 2 ? 1 : 0;
  for (int r = 0; r < world; ++r) {
    a.tp_dst[r] = reinterpret_cast<float*>(s->tp_peer[r] + tp_recv_offset(s, b, me));
    a.tp_flag[r] = reinterpret_cast<unsigned long long*>(s->tp_peer[r] + tp_flag_offset(s, 0, b, me));
  }
  TRY(run_wide(s, mA, mB128, mB256, a));
  TpStep t;
  memset(&t, 0, sizeof(t));
  t.h = s->h;
  t.recv = reinterpret_cast<const float*>(s->tp_buf + tp_recv_offset(s, b, 0));
  t.slot = static_cast<int64_t>(tp_slot(s));
  for (int r = 0; r < world; ++r) {
    t.ag_dst[r] = reinterpret_cast<__nv_bfloat16*>(s->tp_peer[r] + tp_ag_offset(s, b));
    t.ag_flag_of_rank[r] = reinterpret_cast<unsigned long long*>(s->tp_peer[r] + tp_flag_offset(s, 1, b, me));
  }
  t.ag = reinterpret_cast<const __nv_bfloat16*>(s->tp_buf + tp_ag_offset(s, b));
  t.rs_flags = reinterpret_cast<const unsigned long long*>(s->tp_buf + tp_flag_offset(s, 0, b, 0));
  t.ag_flags = reinterpret_cast<const unsigned long long*>(s->tp_buf + tp_flag_offset(s, 1, b, 0));
  t.count = s->tp_count + 2 + b;
  t.epoch = s->tp_epoch;
  t.tag = tag;
  t.world = world;
  t.rank = me;
  t.rows = rows;
  t.H = m->H;
  t.status = s->status;
  const int64_t groups = static_cast<int64_t>(rows) * m->H / 4;
  const unsigned blocks = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>((groups + 255) / 256, s->sms * 4)));
  if (a.tp_all) {
    CK(launch_k(tp_reduce_all_kernel, dim3(blocks), dim3(256), 0, s->stream, true, t));
  } else {
    CK(launch_k(tp_rs_kernel, dim3(blocks), dim3(256), 0, s->stream, true, t));
    CK(launch_k(tp_ag_kernel, dim3(blocks), dim3(256), 0, s->stream, true, t));
  }
  return DRT_OK;
}

// Vocabulary-parallel lm_head over peer memory: this rank projects its vocabulary tiles of the
// final-norm rows (s->xf) and the epilogue stores each logit tile, rounded as the single-GPU head
// rounds it, into every rank's logits at the tile's vocabulary columns (EPI_TP_GATHER); the last
// CTA raises this rank's lm_head flag on every rank, and tp_gather_wait_kernel holds the selector
// until every rank's flag is up. Every rank then holds the whole [rows][V] logits, equal bit for
// bit to one GPU's (each logit is computed once, by the same arithmetic), and runs the selector on
// them. A rank overwrites a peer's logits only in the next step's head, after the peer's layer
// reductions of that step, which follow its selector in stream order.
int tp_gather_head(drt_session* s, int rows, const int* rows_dev) {
  drt_model* m = s->m;
  const int world = m->shard.world, me = m->shard.rank;
  Fwd f = {};
  f.rows = rows;
  f.rows_dev = rows_dev;
  GemmArgs a = base_args(s, s->lm_tiles * 128, m->H, f);
  a.epi = EPI_TP_GATHER;
  a.ld_out = m->V;
  a.tp_world = world;
  a.tp_tag = 2 * m->L;
  a.tp_count = s->tp_count + 4;
  a.tp_epoch = s->tp_epoch;
  for (int r = 0; r < world; ++r) {
    a.tp_dst[r] = reinterpret_cast<float*>(s->tp_peer[r] + tp_logits_offset(s)) + static_cast<size_t>(s->lm_t0) * 128;
    a.tp_flag[r] = reinterpret_cast<unsigned long long*>(s->tp_peer[r] + tp_flag_offset(s, 2, 0, me));
  }
  TRY(run_wide(s, s->m_lm_shard, s->m_xf128, s->head_cap >= 256 ? &s->m_xf256 : nullptr, a));
  TpStep t;
  memset(&t, 0, sizeof(t));
  t.rs_flags = reinterpret_cast<const unsigned long long*>(s->tp_buf + tp_flag_offset(s, 2, 0, 0));
  t.epoch = s->tp_epoch;
  t.tag = 2 * m->L;
  t.world = world;
  t.rank = me;
  t.status = s->status;
  CK(launch_k(tp_gather_wait_kernel, dim3(1), dim3(32), 0, s->stream, true, t));
  return DRT_OK;
}

// Tensor parallelism: sum the ranks' f32 linear partials (s->part, rows x H) over the group, then
// h += bf16(sum), the linear's output rounding applied once to the reduced value.
int tp_reduce_residual(drt_session* s, int rows) {
  drt_model* m = s->m;
  const NcclApi* nc = nullptr;
  TRY(nccl_api(&nc));
  const size_t n = static_cast<size_t>(rows) * m->H;
  NCCL_CK(nc, nc->all_reduce(s->part, s->part, n, ncclFloat32, ncclSum, m->comm, s->stream));
  const unsigned blocks = static_cast<unsigned>(std::min<size_t>((n / 4 + 255) / 256, static_cast<size_t>(s->sms) * 8));
  CK(launch_k(resid_add_bf16r_kernel, dim3(std::max(1u, blocks)), dim3(256), 0, s->stream, false, s->h,
              static_cast<const float*>(s->part), static_cast<int64_t>(n)));
  return DRT_OK;
}

// Enqueue the transformer layers for the rows described by f (embedding through the last
// layer's residual). K/V of every forwarded row is written into the cache.
int enqueue_layers(drt_session* s, const Fwd& f) {
  drt_model* m = s->m;
  const int H = m->H, qd = m->nq * 128;
  if (s->tp_p2p) CK(launch_k(tp_tick_kernel, dim3(1), dim3(32), 0, s->stream, true, s->tp_epoch));
  CK(launch_k(embed_rows_kernel, dim3(f.rows), dim3(128), 0, s->stream, true, static_cast<const int*>(s->canvas), f.pos0,
              f.pos0_dev, f.rows, f.rows_dev, static_cast<const __nv_bfloat16*>(m->embed), H, s->h, m->V, s->status,
              static_cast<float*>(nullptr)));
  for (int l = 0; l < m->L; ++l) {
    LayerW& w = m->layers[l];
    TRY(run_rmsnorm(s, s->h, nullptr, f.rows, f.rows_dev, w.in_norm, s->xn));
    // QKV + QK-norm + RoPE + K/V cache write.
    GemmArgs a = base_args(s, m->qkv_rows, H, f);
    a.epi = EPI_QKV;
    a.out_bf16 = s->q;
    a.bias = w.bqkv;
    a.qnorm_w = w.q_norm;
    a.knorm_w = w.k_norm;
    a.rope_cos = m->rope_cos;
    a.rope_sin = m->rope_sin;
    a.nq = m->nq;
    a.nkv = m->nkv;
    a.kcache = s->kcache + static_cast<size_t>(l) * m->nkv * s->max_seq * 128;
    a.vtcache = s->vtcache + static_cast<size_t>(l) * m->nkv * 128 * s->max_seq;
    a.max_seq = s->max_seq;
    a.eps = m->cfg.rms_norm_eps;
    if (f.decode) {
      TRY(run_dec_gemm(s, w.m_qkv, s->m_xn64, a, m->quantized ? &w.q_qkv : nullptr, &s->m_xn128));
    } else {
      TRY(run_wide(s, w.m_qkv, s->m_xn128, s->rows_cap >= 256 ? &s->m_xn256 : nullptr, a));
    }
    // Attention.
    AttnArgs t;
    memset(&t, 0, sizeof(t));
    t.nq = m->nq;
    t.nkv = m->nkv;
    t.rep = m->rep;
    t.tile_pos = m->tile_pos;
    t.rows = f.rows;
    t.rows_dev = f.rows_dev;
    t.q_pos0 = f.pos0;
    t.q_pos0_dev = f.pos0_dev;
    t.kv_len = f.kv_len;
    t.kv_len_dev = f.kv_len_dev;
    t.prompt_len = f.prompt_len;
    t.block_size = f.block_size;
    t.bidirectional = f.bidirectional;
    t.kv_plane0 = l * m->nkv;
    t.out = s->attn;
    t.status = s->status;
    t.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(128.0));
    const int qtiles = (f.rows + m->tile_pos - 1) / m->tile_pos;
    if (f.decode && s->da_splits > 0) {
      DecAttnArgs da;
      memset(&da, 0, sizeof(da));
      da.nq = m->nq;
      da.nkv = m->nkv;
      da.rep = m->rep;
      da.rows = std::min(f.rows, 128 / m->rep);
      da.rows_dev = f.rows_dev;
      da.q_pos0 = f.pos0;
      da.q_pos0_dev = f.pos0_dev;
      da.kv_len = f.kv_len;
      da.kv_len_dev = f.kv_len_dev;
      da.prompt_len = f.prompt_len;
      da.block_size = f.block_size;
      da.bidirectional = f.bidirectional;
      da.kv_plane0 = l * m->nkv;
      da.splits = s->da_splits;
      da.cluster_merge = s->da_cluster;
      da.out = s->attn;
      da.part_o = s->da_part_o;
      da.part_ml = s->da_part_ml;
      da.status = s->status;
      da.scale_log2 = t.scale_log2;
      CK(launch_cx(attn_decode_kernel, dim3(s->da_splits, m->nkv), dim3(kDaThreads), kDaSmemBytes, s->stream,
                   s->da_cluster ? s->da_splits : 1, s->m_q,
                   s->m_k64, s->m_v, da));
      if (s->da_splits > 1 && !s->da_cluster)
        CK(launch_k(attn_merge_kernel, dim3(m->nkv, 128 / kDaMergeRows), dim3(128 * kDaMergeRows), 0, s->stream, true,
                    static_cast<const float*>(s->da_part_o), static_cast<const float*>(s->da_part_ml), s->da_splits, m->rep,
                    m->nq, da.rows, da.rows_dev, s->attn));
    } else {
    if (f.decode && qtiles == 1) {
      t.splits = s->attn_splits;
      t.tiles_per_split = s->attn_tps;
      CK(launch_kc(attn_prefix_kernel, dim3(qtiles, m->nkv, t.splits), dim3(128), kAttnSmemBytes, s->stream, true,
                   t.splits, s->m_q, s->m_k, s->m_v, t));
    } else {
      t.splits = 1;
      t.tiles_per_split = (s->max_seq + 127) / 128;
      CK(launch_k(attn_wide_kernel, dim3(qtiles, m->nkv, 1), dim3(kAttnWThreads), kAttnSmemBytes, s->stream, true,
                  s->m_q, s->m_k, s->m_v, t));
    }
    }
    // o_proj + residual (tensor parallel: f32 partial, all-reduce, residual add).
    const bool tp = m->shard.world > 1;
    GemmArgs o = base_args(s, H, qd, f);
    o.epi = tp ? EPI_STORE_RAW : EPI_RESID;
    o.out_f32 = tp ? s->part : s->h;
    o.ld_out = H;
    if (s->tp_p2p) TRY(tp_push_linear(s, w.m_o, s->m_attn128, s->rows_cap >= 256 ? &s->m_attn256 : nullptr, o, 0, 2 * l, f.rows));
    else if (f.decode) TRY(run_dec_gemm(s, w.m_o, s->m_attn64, o, m->quantized ? &w.q_o : nullptr, &s->m_attn128));
    else TRY(run_wide(s, w.m_o, s->m_attn128, s->rows_cap >= 256 ? &s->m_attn256 : nullptr, o));
    if (tp && !s->tp_p2p) TRY(tp_reduce_residual(s, f.rows));
    TRY(run_rmsnorm(s, s->h, nullptr, f.rows, f.rows_dev, w.post_norm, s->xn));
    // gate/up + SwiGLU.
    GemmArgs g = base_args(s, m->gu_rows, H, f);
    g.epi = EPI_SWIGLU;
    g.out_bf16 = s->act;
    g.ld_out = m->I;
    if (f.decode) TRY(run_dec_gemm(s, w.m_gu, s->m_xn64, g, m->quantized ? &w.q_gu : nullptr, &s->m_xn128));
    else TRY(run_wide(s, w.m_gu, s->m_xn128, s->rows_cap >= 256 ? &s->m_xn256 : nullptr, g));
    // down + residual.
    GemmArgs d = base_args(s, H, m->I, f);
    d.epi = tp ? EPI_STORE_RAW : EPI_RESID;
    d.out_f32 = tp ? s->part : s->h;
    d.ld_out = H;
    if (s->tp_p2p) TRY(tp_push_linear(s, w.m_down, s->m_act128, s->rows_cap >= 256 ? &s->m_act256 : nullptr, d, 1, 2 * l + 1, f.rows));
    else if (f.decode) TRY(run_dec_gemm(s, w.m_down, s->m_act64, d, m->quantized ? &w.q_down : nullptr, &s->m_act128));
    else TRY(run_wide(s, w.m_down, s->m_act128, s->rows_cap >= 256 ? &s->m_act256 : nullptr, d));
    if (tp && !s->tp_p2p) TRY(tp_reduce_residual(s, f.rows));
  }
  return DRT_OK;
}

// Final norm over the frontier rows (row_index into the forwarded rows), lm_head, selector.
int enqueue_head(drt_session* s, const int* row_index, int rows, const int* rows_dev, bool with_selector) {
  drt_model* m = s->m;
  TRY(run_rmsnorm(s, s->h, row_index, rows, rows_dev, m->final_norm, s->xf));
  Fwd f = {};
  f.rows = rows;
  f.rows_dev = rows_dev;
  GemmArgs a = base_args(s, m->V, m->H, f);
  a.epi = EPI_STORE_F32;
  a.out_f32 = s->logits;
  a.ld_out = m->V;
  TRY(run_dec_gemm(s, m->m_lm, s->m_xf64, a, m->quantized ? &m->q_lm : nullptr, &s->m_xf128));
  if (with_selector) {
    SelArgs sa;
    memset(&sa, 0, sizeof(sa));
    sa.logits = s->logits;
    sa.ld = m->V;
    sa.rows = rows;
    sa.rows_dev = rows_dev;
    sa.vocab = m->V;
    sa.chunk = kSelChunk;
    sa.nchunks = s->sel_chunks;
    sa.mode = SEL_MAXPROB;
    sa.exclude = -1;
    sa.exclude_dev = &s->state->exclude_token;
    sa.part_max = s->sel_pmax;
    sa.part_idx = s->sel_pidx;
    sa.part_sum = s->sel_psum;
    sa.counters = s->sel_cnt;
    sa.row_amax = s->sel_amax;
    sa.row_sum = s->sel_sum;
    sa.conf = s->conf;
    sa.token = s->token;
    sa.status = s->status;
    // Temperature sampling when the request asks for it (read on the device, so one graph serves both).
    sa.sample_t_dev = &s->state->sample_t;
    sa.sample_seed_dev = &s->state->sample_seed;
    sa.sample_forward_dev = &s->state->forward_count;
    sa.positions = s->state->frontier_pos;
    sa.part_skey = s->sel_skey;
    sa.part_skey2 = s->sel_skey2;
    sa.part_sidx = s->sel_sidx;
    sa.row_tie = s->row_tie;
    if (s->cap_sample)
      CK(launch_k(sel_pass1_kernel<true>, dim3(s->sel_chunks, rows), dim3(kSelThreads), 0, s->stream, true, sa));
    else
      CK(launch_k(sel_pass1_kernel<false>, dim3(s->sel_chunks, rows), dim3(kSelThreads), 0, s->stream, true, sa));
  }
  return DRT_OK;
}

Fwd decode_fwd(drt_session* s) {
  Fwd f = {};
  f.decode = true;
  f.rows = kMaxFwdRows;
  f.rows_dev = &s->state->fwd_rows;
  f.pos0_dev = &s->state->fwd_pos0;
  f.kv_len = s->max_seq;
  f.kv_len_dev = &s->state->kv_len;
  f.prompt_len = s->origin;
  f.block_size = s->block_size;
  f.bidirectional = 0;
  return f;
}

int capture(drt_session* s, bool with_policy, cudaGraphExec_t* out) {
  cudaGraph_t graph = nullptr;
  CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  int rc = DRT_OK;
  if (with_policy) {
    if (launch_k(plan_kernel, dim3(1), dim3(32), 0, s->stream, true, s->state, static_cast<const int*>(s->canvas)) != cudaSuccess)
      rc = set_error(DRT_INTERNAL_ERROR, "plan launch failed");
  }
  if (rc == DRT_OK) rc = enqueue_layers(s, decode_fwd(s));
  if (rc == DRT_OK) rc = enqueue_head(s, s->state->frontier_row, kMaxFrontier, &s->state->n_frontier, true);
  if (rc == DRT_OK && with_policy) {
    if (launch_k(commit_kernel, dim3(1), dim3(32), 0, s->stream, true, s->state, s->canvas, static_cast<const double*>(s->conf),
                 static_cast<const int*>(s->token), static_cast<const int*>(s->row_tie), s->trace) != cudaSuccess)
      rc = set_error(DRT_INTERNAL_ERROR, "commit launch failed");
  }
  cudaError_t e = cudaStreamEndCapture(s->stream, &graph);
  if (rc != DRT_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return set_error(DRT_INTERNAL_ERROR, "graph capture failed: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(out, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return set_error(DRT_INTERNAL_ERROR, "graph instantiate failed: %s", cudaGetErrorString(e));
  return DRT_OK;
}

// Prefill rows [p0, p1) (positions whose tokens are final) into the K/V cache, in chunks.
// A quantized model runs every forward through the decode linears (the quantized weights have no wide
// prefill kernel), in chunks of at most kMaxFwdRows rows.
int forward_chunk_rows(const drt_session* s) { return s->m->quantized ? kMaxFwdRows : s->rows_cap; }

int prefill(drt_session* s, int p0, int p1, int prompt_len, int block_size, int bidirectional) {
  const int step = forward_chunk_rows(s);
  for (int c0 = p0; c0 < p1; c0 += step) {
    Fwd f = {};
    f.decode = s->m->quantized;
    f.rows = std::min(step, p1 - c0);
    f.pos0 = c0;
    f.kv_len = c0 + f.rows;
    f.prompt_len = prompt_len;
    f.block_size = block_size;
    f.bidirectional = bidirectional;
    TRY(enqueue_layers(s, f));
    s->m_prefill_rows += f.rows;
  }
  return DRT_OK;
}

constexpr double kToppTieRel = 9.313225746154785e-10;  // 2^-30: nucleus-mass certification bound

// One entropy_count step as a graph: plan (frontier, transfer), the whole canvas forwarded with
// bidirectional attention, final norm over the shifted rows of the frontier, lm_head, top-p
// entropy selector and the top-k commit. Shapes are static; the frontier count lives on the device.
int capture_dream(drt_session* s, const DreamState& g, double temperature, double top_p, cudaGraphExec_t* out) {
  drt_model* m = s->m;
  const int gen_cap = g.canvas_len - g.prompt_len;
  cudaGraph_t graph = nullptr;
  CK(cudaStreamBeginCapture(s->stream, cudaStreamCaptureModeThreadLocal));
  int rc = DRT_OK;
  if (launch_k(dream_plan_kernel, dim3(1), dim3(kDreamThreads), 0, s->stream, true, s->dstate,
               static_cast<const int*>(s->canvas), s->d_fpos, s->scope_rows, static_cast<const int*>(s->d_klist)) != cudaSuccess)
    rc = set_error(DRT_INTERNAL_ERROR, "plan launch failed");
  if (rc == DRT_OK) {
    Fwd f = {};
    f.rows = g.canvas_len;
    f.pos0 = 0;
    f.kv_len = g.canvas_len;
    f.prompt_len = 0;
    f.block_size = 1;
    f.bidirectional = 1;
    rc = enqueue_layers(s, f);
  }
  const int* n_dev = &s->dstate->n_frontier;
  if (rc == DRT_OK) rc = run_rmsnorm(s, s->h, s->scope_rows, gen_cap, n_dev, m->final_norm, s->xf);
  if (rc == DRT_OK) {
    Fwd f = {};
    f.rows = gen_cap;
    f.rows_dev = n_dev;
    if (s->tp_p2p && s->tp_vocab) {
      rc = tp_gather_head(s, gen_cap, n_dev);
    } else {
      GemmArgs a = base_args(s, m->V, m->H, f);
      a.epi = EPI_STORE_F32;
      a.out_f32 = s->logits;
      a.ld_out = m->V;
      rc = run_wide(s, m->m_lm, s->m_xf128, s->head_cap >= 256 ? &s->m_xf256 : nullptr, a);
    }
  }
  if (rc == DRT_OK) {
    ToppArgs t;
    memset(&t, 0, sizeof(t));
    t.logits = s->logits;
    t.ld = m->V;
    t.rows = gen_cap;
    t.rows_dev = n_dev;
    t.vocab = m->V;
    t.temperature = temperature;
    t.top_p = top_p;
    t.exclude = (g.mask_id >= 0 && g.mask_id < m->V) ? g.mask_id : -1;
    t.tie_rel = kToppTieRel;
    t.conf = s->conf;
    t.token = s->token;
    t.tie = s->row_tie;
    if (launch_k(sel_topp_entropy_kernel, dim3(gen_cap), dim3(kToppThreads), kToppSmemBytes, s->stream, true, t) != cudaSuccess)
      rc = set_error(DRT_INTERNAL_ERROR, "selector launch failed");
  }
  if (rc == DRT_OK &&
      launch_k(dream_commit_kernel, dim3(1), dim3(kDreamThreads), 0, s->stream, true, s->dstate, s->canvas,
               static_cast<const int*>(s->d_fpos), static_cast<const double*>(s->conf), static_cast<const int*>(s->token),
               static_cast<const int*>(s->row_tie), kTieRel, static_cast<const int*>(s->d_stepof), s->trace) != cudaSuccess)
    rc = set_error(DRT_INTERNAL_ERROR, "commit launch failed");
  cudaError_t e = cudaStreamEndCapture(s->stream, &graph);
  if (rc != DRT_OK) {
    if (graph) cudaGraphDestroy(graph);
    return rc;
  }
  if (e != cudaSuccess) return set_error(DRT_INTERNAL_ERROR, "graph capture failed: %s", cudaGetErrorString(e));
  e = cudaGraphInstantiate(out, graph, 0);
  cudaGraphDestroy(graph);
  if (e != cudaSuccess) return set_error(DRT_INTERNAL_ERROR, "graph instantiate failed: %s", cudaGetErrorString(e));
  return DRT_OK;
}

// linspace(1, eps, steps + 1) in float64 cast to float32, as NumPy computes it: y = i * step,
// y += 1, the last entry set to eps (numpy/_core/function_base.py linspace).
void entropy_count_timesteps(int steps, double eps, std::vector<float>* ts) {
  ts->assign(steps + 1, 0.0f);
  const double step = (eps - 1.0) / static_cast<double>(steps);
  for (int i = 0; i <= steps; ++i) {
    volatile double y = static_cast<double>(i) * step;  // two roundings, as NumPy's two array ops
    (*ts)[i] = static_cast<float>(y + 1.0);
  }
  (*ts)[steps] = static_cast<float>(eps);
}

void entropy_count_plan(int n_masked, int steps, double eps, int* transfer) {
  std::vector<float> ts;
  entropy_count_timesteps(steps, eps, &ts);
  int n = n_masked;
  for (int i = 0; i < steps; ++i) {
    int k = 0;
    if (n > 0) {
      if (i < steps - 1) {
        const double t = static_cast<double>(ts[i]), u = static_cast<double>(ts[i + 1]);
        const double want = static_cast<double>(n) * (1.0 - u / t);
        k = want >= static_cast<double>(n) ? n : static_cast<int>(want);
      } else {
        k = n;
      }
      if (k < 0) k = 0;
      n -= k;
    }
    transfer[i] = k;
  }
}

int dream_generate(drt_session* s, const drt_generate_params* p, const int32_t* prompt, int32_t prompt_len, int32_t* out,
                   drt_generate_result* result, drt_step_trace* trace) {
  drt_model* m = s->m;
  REQUIRE(p->steps >= 1, "steps must be >= 1");
  REQUIRE(p->max_tokens >= 1, "max_tokens must be >= 1");
  REQUIRE(prompt_len >= 1, "device generation requires a non-empty prompt");
  const int canvas_len = prompt_len + p->max_tokens;
  REQUIRE(canvas_len <= s->rows_cap && canvas_len <= s->max_seq,
          "full-canvas forward of %d positions exceeds the session capacity (%d rows, %d positions)", canvas_len,
          s->rows_cap, s->max_seq);
  REQUIRE(p->max_tokens <= s->head_cap, "canvas of %d masked positions exceeds the frontier capacity %d", p->max_tokens,
          s->head_cap);
  REQUIRE(std::isfinite(p->temperature) && std::isfinite(p->top_p) && p->top_p > 0.0, "temperature / top_p invalid");
  REQUIRE(std::isfinite(p->eps) && p->eps >= 0.0 && p->eps <= 1.0, "eps must be in [0, 1]");
  REQUIRE(p->mask_token_id >= 0 && p->mask_token_id < m->V, "mask token outside the vocabulary");
  for (int i = 0; i < prompt_len; ++i) {
    REQUIRE(prompt[i] >= 0 && prompt[i] < m->V, "prompt token %d outside the vocabulary", prompt[i]);
    REQUIRE(prompt[i] != p->mask_token_id, "device generation cannot carry MASK in its prompt");
  }
  CK(cudaSetDevice(s->device));
  // schedule: the proceeding steps and their transfer counts
  std::vector<int> transfer(p->steps);
  entropy_count_plan(p->max_tokens, p->steps, p->eps, transfer.data());
  std::vector<int> klist, stepof;
  int iterations = 0, left = p->max_tokens;
  for (int i = 0; i < p->steps && left > 0; ++i) {
    ++iterations;
    if (transfer[i] > 0) {
      klist.push_back(transfer[i]);
      stepof.push_back(i);
      left -= transfer[i];
    }
  }
  const int n_proceed = static_cast<int>(klist.size());
  if (n_proceed > s->d_steps_cap) {
    if (s->d_klist) cudaFree(s->d_klist);
    if (s->d_stepof) cudaFree(s->d_stepof);
    s->d_klist = s->d_stepof = nullptr;
    CK(cudaMalloc(&s->d_klist, sizeof(int) * n_proceed));
    CK(cudaMalloc(&s->d_stepof, sizeof(int) * n_proceed));
    s->d_steps_cap = n_proceed;
    if (s->g_dream) { cudaGraphExecDestroy(s->g_dream); s->g_dream = nullptr; }
  }
  if (p->trace_steps > s->trace_cap) {
    if (s->trace) cudaFree(s->trace);
    s->trace = nullptr;
    CK(cudaMalloc(&s->trace, sizeof(StepTrace) * p->trace_steps));
    s->trace_cap = p->trace_steps;
    if (s->g_dream) { cudaGraphExecDestroy(s->g_dream); s->g_dream = nullptr; }
  }
  DreamState* hs = s->hdstate;
  memset(hs, 0, sizeof(DreamState));
  hs->canvas_len = canvas_len;
  hs->prompt_len = prompt_len;
  hs->mask_id = p->mask_token_id;
  hs->shift = m->cfg.logits_shift ? 1 : 0;
  hs->n_proceed = n_proceed;
  hs->trace_cap = std::min(p->trace_steps, s->trace_cap);
  auto& key = s->g_dream_key;
  if (s->g_dream != nullptr && (key.canvas_len != canvas_len || key.prompt_len != prompt_len ||
                                key.mask_id != p->mask_token_id || key.temperature != p->temperature ||
                                key.top_p != p->top_p || key.trace != s->trace)) {
    cudaGraphExecDestroy(s->g_dream);
    s->g_dream = nullptr;
  }
  if (s->g_dream == nullptr) {
    const int64_t before = g_launches;
    TRY(capture_dream(s, *hs, p->temperature, p->top_p, &s->g_dream));
    s->g_dream_kernels = static_cast<int>(g_launches - before);
    key = {canvas_len, prompt_len, p->mask_token_id, p->temperature, p->top_p, s->trace};
  }
  std::vector<int> canvas(canvas_len, p->mask_token_id);
  std::copy(prompt, prompt + prompt_len, canvas.begin());
  cudaEvent_t e_total0 = nullptr, e_total1 = nullptr, e_dec0 = nullptr, e_dec1 = nullptr;
  CK(cudaEventCreate(&e_total0));
  CK(cudaEventCreate(&e_total1));
  CK(cudaEventCreate(&e_dec0));
  CK(cudaEventCreate(&e_dec1));
  CK(cudaEventRecord(e_total0, s->stream));
  CK(cudaMemcpyAsync(s->canvas, canvas.data(), sizeof(int) * canvas_len, cudaMemcpyHostToDevice, s->stream));
  if (n_proceed > 0) {
    CK(cudaMemcpyAsync(s->d_klist, klist.data(), sizeof(int) * n_proceed, cudaMemcpyHostToDevice, s->stream));
    CK(cudaMemcpyAsync(s->d_stepof, stepof.data(), sizeof(int) * n_proceed, cudaMemcpyHostToDevice, s->stream));
  }
  CK(cudaMemcpyAsync(s->dstate, hs, sizeof(DreamState), cudaMemcpyHostToDevice, s->stream));
  CK(cudaEventRecord(e_dec0, s->stream));
  int rc = DRT_OK;
  const auto host0 = std::chrono::steady_clock::now();
  for (int i = 0; i < n_proceed; ++i) {
    if (cudaGraphLaunch(s->g_dream, s->stream) != cudaSuccess) {
      rc = set_error(DRT_INTERNAL_ERROR, "graph launch failed");
      break;
    }
  }
  const float host_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - host0).count();
  cudaEventRecord(e_dec1, s->stream);
  cudaMemcpyAsync(hs, s->dstate, sizeof(DreamState), cudaMemcpyDeviceToHost, s->stream);
  cudaMemcpyAsync(out, s->canvas, sizeof(int) * canvas_len, cudaMemcpyDeviceToHost, s->stream);
  cudaEventRecord(e_total1, s->stream);
  cudaError_t se = cudaStreamSynchronize(s->stream);
  if (rc == DRT_OK && se != cudaSuccess) rc = set_error(DRT_INTERNAL_ERROR, "decode failed: %s", cudaGetErrorString(se));
  float dec_ms = 0.f, tot_ms = 0.f;
  cudaEventElapsedTime(&dec_ms, e_dec0, e_dec1);
  cudaEventElapsedTime(&tot_ms, e_total0, e_total1);
  cudaEventDestroy(e_dec0);
  cudaEventDestroy(e_dec1);
  cudaEventDestroy(e_total0);
  cudaEventDestroy(e_total1);
  TRY(rc);
  TRY(check_status(s));
  if (trace != nullptr && p->trace_steps > 0) {
    const int nt = std::min(hs->forward_count, std::min(p->trace_steps, s->trace_cap));
    CK(cudaMemcpy(trace, s->trace, sizeof(StepTrace) * nt, cudaMemcpyDeviceToHost));
  }
  if (result) {
    result->forward_count = hs->forward_count;
    result->iteration_count = iterations;
    result->committed_token_count = hs->committed_count;
    result->near_tie_steps = hs->near_tie_steps;
    result->exact_tie_steps = hs->exact_tie_steps;
    result->stopped = left == 0 ? 1 : 0;
    result->canvas_len = canvas_len;
    result->prefill_ms = 0.f;
    result->decode_ms = dec_ms;
    result->total_ms = tot_ms;
    result->kernel_launches = n_proceed * s->g_dream_kernels;
    result->host_enqueue_ms = host_ms;
  }
  s->m_forwards += hs->forward_count;
  s->m_rows += static_cast<int64_t>(hs->forward_count) * canvas_len;
  s->m_committed += hs->committed_count;
  s->m_near += hs->near_tie_steps;
  s->m_exact += hs->exact_tie_steps;
  s->m_ms += dec_ms;
  s->started = false;
  return DRT_OK;
}
}  // namespace

extern "C" int drt_session_open(drt_model* m, const drt_session_config* cfg, drt_session** out) {
  REQUIRE(m && cfg && out, "null argument");
  *out = nullptr;
  const bool dream = cfg->decode_strategy == DRT_STRATEGY_ENTROPY_COUNT;
  REQUIRE(dream || cfg->decode_strategy == DRT_STRATEGY_BD3_FIXED_QUOTA || cfg->decode_strategy == DRT_STRATEGY_BLOCK_THRESHOLD ||
              cfg->decode_strategy == DRT_STRATEGY_D2F_BLOCK_PIPELINE,
          "device sessions run only block_threshold, d2f_block_pipeline, bd3_fixed_quota and entropy_count (got strategy %d)",
          cfg->decode_strategy);
  REQUIRE(dream || m->shard.world == 1, "a tensor-parallel model serves entropy_count sessions only");
  if (dream) {
    REQUIRE(cfg->attention_mask_kind == DRT_MASK_BIDIRECTIONAL, "entropy_count sessions serve the bidirectional graph only");
    REQUIRE(!m->quantized, "entropy_count sessions need bf16 linears (the quantized path forwards at most %d rows)", kMaxFwdRows);
  } else {
    REQUIRE(cfg->attention_mask_kind == DRT_MASK_D2F_HYBRID, "this device session serves the d2f_hybrid graph only");
    REQUIRE(cfg->block_size >= 1 && cfg->block_size <= 32, "block_size must be in [1, 32]");
  }
  CK(cudaSetDevice(m->device));
  drt_session* s = new drt_session();
  s->m = m;
  s->cfg = *cfg;
  s->device = m->device;
  s->max_seq = ((m->cfg.max_seq + 127) / 128) * 128;
  s->rows_cap = std::max(64, ((std::max(m->cfg.max_prefill_rows, 64) + 127) / 128) * 128);
  s->planes = m->L * m->nkv;
  s->sms = num_sms(m->device);
  s->dream = dream;
  s->head_cap = dream ? std::min(s->rows_cap, kDreamMaxFrontier) : kMaxFrontier;
  auto fail = [&](int rc) { drt_session_close(s); return rc; };
  int rc;
  if (cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking) != cudaSuccess) return fail(set_error(DRT_INTERNAL_ERROR, "stream create failed"));
  if (cudaEventCreate(&s->ev0) != cudaSuccess || cudaEventCreate(&s->ev1) != cudaSuccess) return fail(set_error(DRT_INTERNAL_ERROR, "event create failed"));
  const int H = m->H, qd = m->nq * 128, R = s->rows_cap;
  if ((rc = salloc(s, &s->canvas, s->max_seq)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->h, static_cast<size_t>(R) * H)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->xn, static_cast<size_t>(R) * H)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->q, static_cast<size_t>(R) * qd)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->attn, static_cast<size_t>(R) * qd)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->act, static_cast<size_t>(R) * m->I)) != DRT_OK) return fail(rc);
  const int xf_rows = std::max(s->head_cap, 128);  // the final-norm rows, at least one 128-row box
  if ((rc = salloc(s, &s->xf, static_cast<size_t>(xf_rows) * H)) != DRT_OK) return fail(rc);
  // stream-K workspace (one 128 x 128 f32 partial per SM) and its flags
  if ((rc = salloc(s, &s->sk_part, static_cast<size_t>(s->sms) * 128 * 128)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sk_flag, static_cast<size_t>(s->sms))) != DRT_OK) return fail(rc);
  if (cudaMemset(s->sk_flag, 0, sizeof(int) * s->sms) != cudaSuccess) return fail(set_error(DRT_INTERNAL_ERROR, "memset failed"));
  // a tensor-parallel session's logits live in its peer-mapped buffer (below): with the
  // vocabulary-parallel lm_head every rank's projection stores its tiles there
  if (m->shard.world <= 1 && (rc = salloc(s, &s->logits, static_cast<size_t>(s->head_cap) * m->V)) != DRT_OK) return fail(rc);
  if (m->shard.world > 1) {
    if ((rc = salloc(s, &s->part, static_cast<size_t>(R) * H)) != DRT_OK) return fail(rc);
    const size_t bytes = tp_buf_bytes(s);
    if ((rc = salloc(s, &s->tp_buf, bytes)) != DRT_OK) return fail(rc);
    s->logits = reinterpret_cast<float*>(s->tp_buf + tp_logits_offset(s));
    if ((rc = salloc(s, &s->tp_count, 5)) != DRT_OK) return fail(rc);
    if ((rc = salloc(s, &s->tp_epoch, 1)) != DRT_OK) return fail(rc);
    if (cudaMemset(s->tp_buf, 0, bytes) != cudaSuccess || cudaMemset(s->tp_count, 0, 5 * sizeof(int)) != cudaSuccess ||
        cudaMemset(s->tp_epoch, 0, sizeof(unsigned long long)) != cudaSuccess)
      return fail(set_error(DRT_INTERNAL_ERROR, "memset failed"));
  }
  const size_t kv = static_cast<size_t>(s->planes) * s->max_seq * 128;
  if ((rc = salloc(s, &s->kcache, kv)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->vtcache, kv)) != DRT_OK) return fail(rc);
  if (cudaMemset(s->kcache, 0, kv * 2) != cudaSuccess || cudaMemset(s->vtcache, 0, kv * 2) != cudaSuccess)
    return fail(set_error(DRT_INTERNAL_ERROR, "kv memset failed"));
  // Largest cluster the GPU co-schedules for the split kernels (16 needs the non-portable
  // opt-in; fall back to 8).
  {
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(1, 1, 16);
    lc.blockDim = dim3(128);
    lc.dynamicSmemBytes = kAttnSmemBytes;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeClusterDimension;
    at[0].val.clusterDim.x = 1;
    at[0].val.clusterDim.y = 1;
    at[0].val.clusterDim.z = 16;
    lc.attrs = at;
    lc.numAttrs = 1;
    int n16 = 0;
    if (cudaOccupancyMaxActiveClusters(&n16, attn_prefix_kernel, &lc) != cudaSuccess || n16 < 1) {
      cudaGetLastError();
      s->max_cluster = 8;
    }
  }
  // Split-KV attention for one decode query tile: a power-of-two cluster of 4..16 CTAs per head.
  const int kv_tiles = (s->max_seq + 127) / 128;
  int asp = 1;
  while (asp < s->max_cluster && asp < kv_tiles && m->nkv * asp < (s->sms * 4) / 5) asp *= 2;
  if (asp == 2) asp = kv_tiles >= 4 ? 4 : 1;
  s->attn_splits = asp;
  s->attn_tps = (kv_tiles + asp - 1) / asp;
  // Decode attention: enough CTAs per KV head that each covers at most kDaMaxSub 64-key sub-tiles
  // of the longest canvas (one CTA per SM; without the cluster merge the CTAs wait on nothing, so a
  // long canvas may take more than one wave); otherwise the general kernel.
  {
    const int n_sub = (s->max_seq + 63) / 64;  // sub-tiles of the longest canvas, the last one partial
    const int sp = (n_sub + kDaMaxSub - 1) / kDaMaxSub;
    // every forwarded row of a decode forward (up to kMaxFwdRows: a finished block forwarded again
    // plus the window) times the query heads per KV head must fit the kernel's 128 UMMA rows
    const bool fits = m->rep * kMaxFwdRows <= 128 && sp <= kDaMaxSplits;
    s->da_splits = fits ? sp : 0;
    // One cluster per KV head when every cluster can be resident at once: the split merge then
    // happens in distributed shared memory instead of a second kernel.
    if (s->da_splits > 1 && s->da_splits <= 16) {
      cudaLaunchConfig_t lc = {};
      lc.gridDim = dim3(s->da_splits, m->nkv);
      lc.blockDim = dim3(kDaThreads);
      lc.dynamicSmemBytes = kDaSmemBytes;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = static_cast<unsigned>(s->da_splits);
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      lc.attrs = at;
      lc.numAttrs = 1;
      int nc = 0;
      if (cudaOccupancyMaxActiveClusters(&nc, attn_decode_kernel, &lc) != cudaSuccess) {
        cudaGetLastError();
        nc = 0;
      }
      s->da_cluster = nc >= m->nkv ? 1 : 0;
    }
    if (s->da_splits > 1 && !s->da_cluster) {
      const size_t rows = static_cast<size_t>(m->nkv) * s->da_splits * 128;
      if ((rc = salloc(s, &s->da_part_o, rows * 128)) != DRT_OK) return fail(rc);
      if ((rc = salloc(s, &s->da_part_ml, rows * 2)) != DRT_OK) return fail(rc);
    }
  }
  // Selector scratch.
  s->sel_chunks = (m->V + kSelChunk - 1) / kSelChunk;
  const size_t np = static_cast<size_t>(kMaxFrontier) * s->sel_chunks;
  if ((rc = salloc(s, &s->sel_pmax, np)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sel_pidx, np)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sel_psum, np)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sel_cnt, kMaxFrontier)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sel_skey, np)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sel_skey2, np)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sel_sidx, np)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sel_amax, kMaxFrontier)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->sel_sum, kMaxFrontier)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->conf, s->head_cap)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->token, s->head_cap)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->scope_rows, s->head_cap)) != DRT_OK) return fail(rc);
  if (cudaMemset(s->sel_cnt, 0, sizeof(int) * kMaxFrontier) != cudaSuccess) return fail(set_error(DRT_INTERNAL_ERROR, "memset failed"));
  if ((rc = salloc(s, &s->row_tie, s->head_cap)) != DRT_OK) return fail(rc);
  if (dream) {
    if ((rc = salloc(s, &s->d_fpos, s->head_cap)) != DRT_OK) return fail(rc);
    if ((rc = salloc(s, &s->dstate, 1)) != DRT_OK) return fail(rc);
    if (cudaMallocHost(&s->hdstate, sizeof(DreamState)) != cudaSuccess) return fail(set_error(DRT_INTERNAL_ERROR, "pinned alloc failed"));
    if (s->head_cap >= 256 && (rc = map_matrix(&s->m_xf256, s->xf, s->head_cap, H, 256)) != DRT_OK) return fail(rc);
  }
  if ((rc = salloc(s, &s->status, 1)) != DRT_OK) return fail(rc);
  if ((rc = salloc(s, &s->state, 1)) != DRT_OK) return fail(rc);
  if (cudaMemset(s->status, 0, sizeof(int)) != cudaSuccess || cudaMemset(s->state, 0, sizeof(DecodeState)) != cudaSuccess)
    return fail(set_error(DRT_INTERNAL_ERROR, "memset failed"));
  if (cudaMallocHost(&s->hstate, sizeof(DecodeState)) != cudaSuccess || cudaMallocHost(&s->hflags, sizeof(int) * 8) != cudaSuccess)
    return fail(set_error(DRT_INTERNAL_ERROR, "pinned alloc failed"));
  memset(s->hstate, 0, sizeof(DecodeState));
  // Tensor maps over the activation buffers and the K/V cache.
  if ((rc = map_matrix(&s->m_xn64, s->xn, R, H, 64)) != DRT_OK) return fail(rc);
  if ((rc = map_matrix(&s->m_xn128, s->xn, R, H, 128)) != DRT_OK) return fail(rc);
  if (R >= 256 && (rc = map_matrix(&s->m_xn256, s->xn, R, H, 256)) != DRT_OK) return fail(rc);
  if (R >= 256 && (rc = map_matrix(&s->m_attn256, s->attn, R, qd, 256)) != DRT_OK) return fail(rc);
  if (R >= 256 && (rc = map_matrix(&s->m_act256, s->act, R, m->I, 256)) != DRT_OK) return fail(rc);
  if ((rc = map_matrix(&s->m_attn64, s->attn, R, qd, 64)) != DRT_OK) return fail(rc);
  if ((rc = map_matrix(&s->m_attn128, s->attn, R, qd, 128)) != DRT_OK) return fail(rc);
  if ((rc = map_matrix(&s->m_act64, s->act, R, m->I, 64)) != DRT_OK) return fail(rc);
  if ((rc = map_matrix(&s->m_act128, s->act, R, m->I, 128)) != DRT_OK) return fail(rc);
  if ((rc = map_matrix(&s->m_xf64, s->xf, s->head_cap, H, 64)) != DRT_OK) return fail(rc);
  if ((rc = map_matrix(&s->m_xf128, s->xf, xf_rows, H, 128)) != DRT_OK) return fail(rc);
  {
    const uint64_t dq[3] = {128, static_cast<uint64_t>(m->nq), static_cast<uint64_t>(R)};
    const uint64_t sq[2] = {256, static_cast<uint64_t>(qd) * 2};
    const uint32_t bq[3] = {64, static_cast<uint32_t>(m->rep), static_cast<uint32_t>(m->tile_pos)};
    if ((rc = make_map(&s->m_q, s->q, 3, dq, sq, bq)) != DRT_OK) return fail(rc);
    const uint64_t dk[3] = {128, static_cast<uint64_t>(s->max_seq), static_cast<uint64_t>(s->planes)};
    const uint64_t sk[2] = {256, static_cast<uint64_t>(s->max_seq) * 256};
    const uint32_t bk[3] = {64, 128, 1};
    if ((rc = make_map(&s->m_k, s->kcache, 3, dk, sk, bk)) != DRT_OK) return fail(rc);
    const uint32_t bk64[3] = {64, 64, 1};
    if ((rc = make_map(&s->m_k64, s->kcache, 3, dk, sk, bk64)) != DRT_OK) return fail(rc);
    const uint64_t dv[3] = {static_cast<uint64_t>(s->max_seq), 128, static_cast<uint64_t>(s->planes)};
    const uint64_t sv[2] = {static_cast<uint64_t>(s->max_seq) * 2, static_cast<uint64_t>(s->max_seq) * 256};
    const uint32_t bv[3] = {64, 128, 1};
    if ((rc = make_map(&s->m_v, s->vtcache, 3, dv, sv, bv)) != DRT_OK) return fail(rc);
  }
  if (cudaDeviceSynchronize() != cudaSuccess) return fail(set_error(DRT_INTERNAL_ERROR, "session init failed"));
  *out = s;
  return DRT_OK;
}

extern "C" void drt_session_close(drt_session* s) {
  if (!s) return;
  cudaSetDevice(s->device);
  if (s->stream) cudaStreamSynchronize(s->stream);
  if (s->g_step) cudaGraphExecDestroy(s->g_step);
  if (s->g_fwd) cudaGraphExecDestroy(s->g_fwd);
  if (s->g_dream) cudaGraphExecDestroy(s->g_dream);
  for (int r = 0; r < kTpMaxRanks; ++r)
    if (s->tp_peer[r] != nullptr && s->tp_peer[r] != s->tp_buf) cudaIpcCloseMemHandle(s->tp_peer[r]);
  for (void* p : s->allocs) cudaFree(p);
  if (s->d_klist) cudaFree(s->d_klist);
  if (s->d_stepof) cudaFree(s->d_stepof);
  if (s->hdstate) cudaFreeHost(s->hdstate);
  if (s->trace) cudaFree(s->trace);
  if (s->hstate) cudaFreeHost(s->hstate);
  if (s->hflags) cudaFreeHost(s->hflags);
  if (s->ev0) cudaEventDestroy(s->ev0);
  if (s->ev1) cudaEventDestroy(s->ev1);
  if (s->stream) cudaStreamDestroy(s->stream);
  delete s;
}

extern "C" int drt_session_kv_pointers(drt_session* s, void** k, void** v) {
  REQUIRE(s, "null session");
  if (k) *k = s->kcache;
  if (v) *v = s->vtcache;
  return DRT_OK;
}

extern "C" int drt_session_start(drt_session* s, const int32_t* x, int32_t n, int32_t prompt_len, int32_t block_size,
                                 int32_t mask_token_id, int32_t exact_kv, int32_t steps, int64_t memory_budget_bytes,
                                 double temperature, uint64_t seed) {
  REQUIRE(s && x, "null argument");
  // The reference refuses exact K/V on a bidirectional canvas (device_runtime.py:125-126); this
  // build's bidirectional (entropy_count) sessions decode through drt_session_generate only.
  REQUIRE(!(s->dream && exact_kv), "bidirectional device generation cannot use exact D2F K/V");
  if (s->dream)
    return set_error(DRT_UNSUPPORTED, "an entropy_count session decodes through generate; the bidirectional "
                                      "propose route (fixed_quota) is not served");
  REQUIRE(n > 0 && n <= s->max_seq, "canvas length %d outside [1, %d]", n, s->max_seq);
  REQUIRE(prompt_len >= 0 && prompt_len <= n, "prompt_len outside the canvas");
  REQUIRE(block_size >= 1 && block_size <= 32, "block_size must be in [1, 32]");
  REQUIRE(steps >= 1, "steps must be >= 1");
  REQUIRE(memory_budget_bytes >= 0, "memory_budget_bytes must be >= 0");
  REQUIRE(std::isfinite(temperature) && temperature >= 0.0, "temperature must be finite and >= 0");
  // Above temperature 0 the fixed-quota policy draws each row's token (TopConfidence with sampling,
  // diffusion_runtime.py:796-828); the threshold policy refuses a temperature (device_runtime.py:207-213).
  REQUIRE(temperature == 0.0 || s->cfg.decode_strategy == DRT_STRATEGY_BD3_FIXED_QUOTA,
          "the block_threshold policy scores at temperature 0 only");
  if (memory_budget_bytes > 0 && memory_budget_bytes < s->bytes + s->m->bytes)
    return set_error(DRT_INVALID_ARGUMENT, "memory budget %lld below the session's %lld device bytes",
                     static_cast<long long>(memory_budget_bytes), static_cast<long long>(s->bytes + s->m->bytes));
  for (int i = 0; i < n; ++i) REQUIRE(x[i] >= 0 && x[i] < s->m->V, "token %d at position %d outside the vocabulary", x[i], i);
  CK(cudaSetDevice(s->device));
  CK(cudaMemcpyAsync(s->canvas, x, sizeof(int) * n, cudaMemcpyHostToDevice, s->stream));
  memset(s->hstate, 0, sizeof(DecodeState));
  s->hstate->canvas_len = n;
  s->hstate->mask_id = mask_token_id;
  s->hstate->active_block = -1;
  s->hstate->sample_t = temperature;
  s->hstate->sample_seed = seed;
  CK(cudaMemcpyAsync(s->state, s->hstate, sizeof(DecodeState), cudaMemcpyHostToDevice, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  s->canvas_len = n;
  s->origin = prompt_len;
  s->block_size = block_size;
  s->mask_id = mask_token_id;
  s->exact_kv = exact_kv != 0;
  s->propose_count = 0;
  s->started = true;
  return DRT_OK;
}

extern "C" int drt_session_propose(drt_session* s, const int32_t* frontier, int32_t nf, int32_t window_end, int32_t frozen,
                                   double* scores, int32_t* tokens, int32_t* forwarded) {
  REQUIRE(s && frontier && scores && tokens, "null argument");
  REQUIRE(s->started, "propose_device before start_device");
  REQUIRE(!s->dream, "an entropy_count session decodes through generate");
  REQUIRE(nf >= 1 && nf <= kMaxFrontier, "frontier size %d outside [1, %d]", nf, kMaxFrontier);
  REQUIRE(window_end >= 1 && window_end <= s->canvas_len, "window_end %d outside [1, %d]", window_end, s->canvas_len);
  REQUIRE(frozen >= 0 && frozen < window_end, "frozen_prefix %d outside [0, window_end)", frozen);
  REQUIRE(window_end - frozen < kMaxFwdRows, "active window of %d rows exceeds %d", window_end - frozen, kMaxFwdRows - 1);
  for (int i = 0; i < nf; ++i) REQUIRE(frontier[i] >= frozen && frontier[i] < window_end, "frontier position %d outside [%d, %d)", frontier[i], frozen, window_end);
  CK(cudaSetDevice(s->device));
  const int fwd_sample = s->hstate->sample_t > 0.0 ? 1 : 0;
  if (s->g_fwd != nullptr && (s->g_fwd_geom[0] != s->origin || s->g_fwd_geom[1] != s->block_size ||
                              s->g_fwd_geom[2] != fwd_sample)) {
    cudaGraphExecDestroy(s->g_fwd);
    s->g_fwd = nullptr;
  }
  if (s->g_fwd == nullptr) {
    s->cap_sample = fwd_sample;
    TRY(capture(s, false, &s->g_fwd));
    s->g_fwd_geom[0] = s->origin;
    s->g_fwd_geom[1] = s->block_size;
    s->g_fwd_geom[2] = fwd_sample;
  }
  DecodeState* hs = s->hstate;
  // exact_kv: the frozen prefix's K/V from earlier forwards is reused (exact under the block-causal
  // d2f mask, whose frozen rows never attend past the prefix). Without it every forward recomputes
  // the K/V of the whole window, the reference's cache-off shape.
  int cache_end = s->exact_kv ? std::min(hs->cache_end, frozen) : 0;
  CK(cudaEventRecord(s->ev0, s->stream));
  int fwd_rows_total = 0;
  // Final rows that are not cached yet go through the prefill path on the first forward (the prompt,
  // as in drt_session_generate) and when they and the window do not fit one decode forward;
  // otherwise they are forwarded with the window, as the device-resident loop forwards them.
  const int shift_rows = s->m->cfg.logits_shift ? 1 : 0;
  if (frozen > cache_end && (cache_end == 0 || window_end - cache_end + shift_rows > kMaxFwdRows)) {
    TRY(prefill(s, cache_end, frozen, s->origin, s->block_size, 0));
    fwd_rows_total += frozen - cache_end;
    cache_end = frozen;
  }
  // Under dream_ar_shift position p is scored from row p - 1: the row before the frozen boundary
  // (the shift feeder) is forwarded again when nothing earlier is.
  const int shift = s->m->cfg.logits_shift ? 1 : 0;
  const int pos0 = (shift && cache_end > frozen - 1) ? std::max(frozen - 1, 0) : cache_end;
  hs->shift = shift;
  hs->fwd_pos0 = pos0;
  hs->fwd_rows = window_end - pos0;
  hs->kv_len = window_end;
  hs->n_frontier = nf;
  for (int i = 0; i < nf; ++i) {
    hs->frontier_pos[i] = frontier[i];
    hs->frontier_row[i] = std::max(frontier[i] - shift, 0) - pos0;
  }
  hs->cache_end = frozen;
  hs->action = PLAN_PROCEED;
  hs->exclude_token = s->cfg.decode_strategy == DRT_STRATEGY_BD3_FIXED_QUOTA ? -1 : s->mask_id;
  hs->forward_count = s->propose_count;  // the sampled draw's forward index
  fwd_rows_total += hs->fwd_rows;
  CK(cudaMemcpyAsync(s->state, hs, sizeof(DecodeState), cudaMemcpyHostToDevice, s->stream));
  CK(cudaGraphLaunch(s->g_fwd, s->stream));
  CK(cudaEventRecord(s->ev1, s->stream));
  CK(cudaMemcpyAsync(scores, s->conf, sizeof(double) * nf, cudaMemcpyDeviceToHost, s->stream));
  CK(cudaMemcpyAsync(tokens, s->token, sizeof(int) * nf, cudaMemcpyDeviceToHost, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  TRY(check_status(s));
  float ms = 0.f;
  cudaEventElapsedTime(&ms, s->ev0, s->ev1);
  s->m_ms += ms;
  s->m_forwards += 1;
  s->m_rows += fwd_rows_total;
  s->propose_count += 1;
  if (forwarded) *forwarded = fwd_rows_total;
  return DRT_OK;
}

extern "C" int drt_session_commit(drt_session* s, const int32_t* positions, const int32_t* tokens, int32_t n) {
  REQUIRE(s && (n == 0 || (positions && tokens)), "null argument");
  REQUIRE(s->started, "commit_device before start_device");
  CK(cudaSetDevice(s->device));
  for (int i = 0; i < n; ++i) {
    REQUIRE(positions[i] >= 0 && positions[i] < s->canvas_len, "commit position %d outside the canvas", positions[i]);
    REQUIRE(tokens[i] >= 0 && tokens[i] < s->m->V, "commit token %d outside the vocabulary", tokens[i]);
    REQUIRE(positions[i] >= s->hstate->cache_end, "commit position %d is inside the frozen prefix", positions[i]);
  }
  for (int i = 0; i < n; ++i)
    CK(cudaMemcpyAsync(s->canvas + positions[i], tokens + i, sizeof(int), cudaMemcpyHostToDevice, s->stream));
  CK(cudaStreamSynchronize(s->stream));
  s->m_committed += n;
  return DRT_OK;
}

extern "C" int drt_session_execute_window(drt_session* s, const int32_t* token_ids, int32_t n_tokens, const int32_t* scope,
                                          int32_t n_scope, int32_t prompt_len, int32_t block_size, float* logits,
                                          int32_t* forwarded_rows) {
  REQUIRE(s && token_ids && scope && logits, "null argument");
  REQUIRE(n_tokens >= 1 && n_tokens <= s->max_seq, "window length %d outside [1, %d]", n_tokens, s->max_seq);
  REQUIRE(n_scope >= 1, "empty scope");
  REQUIRE(prompt_len >= 0 && prompt_len <= n_tokens && block_size >= 1, "bad mask geometry");
  for (int i = 0; i < n_scope; ++i) REQUIRE(scope[i] >= 0 && scope[i] < n_tokens, "scope position %d outside the window", scope[i]);
  for (int i = 0; i < n_tokens; ++i) REQUIRE(token_ids[i] >= 0 && token_ids[i] < s->m->V, "token outside the vocabulary");
  // A full-canvas (entropy_count) session forwards the window in one bidirectional pass. Under the
  // Dream logits convention (logits_shift) position p reads raw row max(p - 1, 0).
  const bool shift = s->m->cfg.logits_shift != 0;
  if (s->dream)
    REQUIRE(n_tokens <= s->rows_cap, "bidirectional window of %d positions exceeds the session's %d rows", n_tokens,
            s->rows_cap);
  CK(cudaSetDevice(s->device));
  drt_model* m = s->m;
  CK(cudaMemcpyAsync(s->canvas, token_ids, sizeof(int) * n_tokens, cudaMemcpyHostToDevice, s->stream));
  std::vector<int> rows;
  const int step = forward_chunk_rows(s);
  for (int c0 = 0; c0 < n_tokens; c0 += step) {
    Fwd f = {};
    f.decode = m->quantized;
    f.rows = std::min(step, n_tokens - c0);
    f.pos0 = c0;
    f.kv_len = c0 + f.rows;
    f.prompt_len = prompt_len;
    f.block_size = block_size;
    f.bidirectional = s->dream ? 1 : 0;
    TRY(enqueue_layers(s, f));
    // Scope rows whose raw row lies inside this chunk, in scope order, up to 64 per head pass.
    auto raw_row = [&](int p) { return shift ? std::max(p - 1, 0) : p; };
    std::vector<int> idx;
    for (int i = 0; i < n_scope; ++i)
      if (raw_row(scope[i]) >= c0 && raw_row(scope[i]) < c0 + f.rows) idx.push_back(i);
    for (size_t b = 0; b < idx.size(); b += kMaxFrontier) {
      const int cnt = static_cast<int>(std::min<size_t>(kMaxFrontier, idx.size() - b));
      rows.assign(cnt, 0);
      for (int j = 0; j < cnt; ++j) rows[j] = raw_row(scope[idx[b + j]]) - c0;
      CK(cudaMemcpyAsync(s->scope_rows, rows.data(), sizeof(int) * cnt, cudaMemcpyHostToDevice, s->stream));
      TRY(enqueue_head(s, s->scope_rows, cnt, nullptr, false));
      for (int j = 0; j < cnt; ++j)
        CK(cudaMemcpyAsync(logits + static_cast<size_t>(idx[b + j]) * m->V, s->logits + static_cast<size_t>(j) * m->V,
                           sizeof(float) * m->V, cudaMemcpyDeviceToHost, s->stream));
      CK(cudaStreamSynchronize(s->stream));
    }
  }
  CK(cudaStreamSynchronize(s->stream));
  TRY(check_status(s));
  // The session canvas now holds this window; a later device decode must start again.
  s->started = false;
  s->hstate->cache_end = 0;
  s->m_forwards += 1;
  s->m_rows += n_tokens;
  if (forwarded_rows) *forwarded_rows = n_tokens;
  return DRT_OK;
}

extern "C" int drt_session_generate(drt_session* s, const drt_generate_params* p, const int32_t* prompt, int32_t prompt_len,
                                    int32_t* out, drt_generate_result* result, drt_step_trace* trace) {
  REQUIRE(s && p && prompt && out, "null argument");
  if (s->dream) {
    REQUIRE(p->decode_strategy == DRT_STRATEGY_ENTROPY_COUNT, "an entropy_count session generates with entropy_count only");
    return dream_generate(s, p, prompt, prompt_len, out, result, trace);
  }
  const bool pipeline = p->decode_strategy == DRT_STRATEGY_D2F_BLOCK_PIPELINE;
  REQUIRE(p->decode_strategy == DRT_STRATEGY_BD3_FIXED_QUOTA || p->decode_strategy == DRT_STRATEGY_BLOCK_THRESHOLD || pipeline,
          "device generation runs bd3_fixed_quota, block_threshold or d2f_block_pipeline");
  if (pipeline) {
    // D2FBlockPipelineCommit.__post_init__ (diffusion_runtime.py:1500-1550)
    REQUIRE(std::isfinite(p->add_threshold) && p->add_threshold > 0.0 && p->add_threshold <= 1.0,
            "add_threshold (tau_add) must be in (0, 1]");
    REQUIRE(std::isfinite(p->activate_threshold) && p->activate_threshold > 0.0 && p->activate_threshold <= 1.0,
            "activate_threshold (tau_act) must be in (0, 1]");
  }
  REQUIRE(p->block_size >= 1 && p->block_size <= 32, "block_size must be in [1, 32]");
  REQUIRE(p->steps >= 1, "steps must be >= 1");
  REQUIRE(p->max_tokens >= 0, "max_tokens must be >= 0");
  REQUIRE(prompt_len >= 1, "device generation requires a non-empty prompt");
  const int canvas_len = prompt_len + p->max_tokens;
  REQUIRE(canvas_len <= s->max_seq, "canvas of %d positions exceeds the session capacity %d", canvas_len, s->max_seq);
  REQUIRE(std::isfinite(p->confidence_threshold) && p->confidence_threshold >= 0.0 && p->confidence_threshold <= 1.0,
          "confidence_threshold must be finite and in [0, 1]");
  REQUIRE(std::isfinite(p->temperature) && p->temperature >= 0.0, "temperature must be finite and >= 0");
  REQUIRE(p->temperature == 0.0 || p->decode_strategy == DRT_STRATEGY_BD3_FIXED_QUOTA,
          "the block_threshold and d2f_block_pipeline policies score at temperature 0 only");
  if (p->decode_strategy == DRT_STRATEGY_BD3_FIXED_QUOTA)
    REQUIRE(prompt_len % p->block_size == 0, "BD3LM Candidate prompt length must be a multiple of block_size");
  for (int i = 0; i < prompt_len; ++i) {
    REQUIRE(prompt[i] >= 0 && prompt[i] < s->m->V, "prompt token %d outside the vocabulary", prompt[i]);
    REQUIRE(prompt[i] != p->mask_token_id, "device generation cannot carry MASK in its prompt");
  }
  REQUIRE(p->mask_token_id >= 0 && p->mask_token_id < s->m->V, "mask token outside the vocabulary");
  CK(cudaSetDevice(s->device));
  if (p->trace_steps > s->trace_cap) {
    if (s->trace) cudaFree(s->trace);
    s->trace = nullptr;
    CK(cudaMalloc(&s->trace, sizeof(StepTrace) * p->trace_steps));
    s->trace_cap = p->trace_steps;
    if (s->g_step) { cudaGraphExecDestroy(s->g_step); s->g_step = nullptr; }
  }
  // d2f mask origin: 0 for the BD3LM graph's absolute blocks, the prompt length for the D2F graph
  REQUIRE(p->mask_origin >= -1 && p->mask_origin <= prompt_len, "mask_origin outside [-1, prompt_len]");
  s->origin = p->mask_origin < 0 ? prompt_len : p->mask_origin;
  // A frozen pipeline block's K/V are final only if no attention block straddles two pipeline blocks.
  REQUIRE(!pipeline || (prompt_len - s->origin) % p->block_size == 0,
          "d2f_block_pipeline needs prompt_len - mask_origin (%d) to be a multiple of block_size (%d)",
          prompt_len - s->origin, p->block_size);
  s->block_size = p->block_size;
  const int step_sample = p->temperature > 0.0 ? 1 : 0;
  if (s->g_step != nullptr && (s->g_step_geom[0] != s->origin || s->g_step_geom[1] != s->block_size ||
                               s->g_step_geom[2] != step_sample)) {
    cudaGraphExecDestroy(s->g_step);
    s->g_step = nullptr;
  }
  if (s->g_step == nullptr) {
    const int64_t before = g_launches;
    s->cap_sample = step_sample;
    TRY(capture(s, true, &s->g_step));
    s->g_step_kernels = static_cast<int>(g_launches - before);
    s->g_step_geom[0] = s->origin;
    s->g_step_geom[1] = s->block_size;
    s->g_step_geom[2] = step_sample;
  }

  std::vector<int> canvas(canvas_len, p->mask_token_id);
  std::copy(prompt, prompt + prompt_len, canvas.begin());
  cudaEvent_t e_total0 = nullptr, e_total1 = nullptr;
  CK(cudaEventCreate(&e_total0));
  CK(cudaEventCreate(&e_total1));
  CK(cudaEventRecord(e_total0, s->stream));
  CK(cudaMemcpyAsync(s->canvas, canvas.data(), sizeof(int) * canvas_len, cudaMemcpyHostToDevice, s->stream));
  DecodeState* hs = s->hstate;
  memset(hs, 0, sizeof(DecodeState));
  hs->canvas_len = canvas_len;
  hs->prompt_len = prompt_len;
  hs->gen_len = p->max_tokens;
  hs->block_size = p->block_size;
  hs->mask_id = p->mask_token_id;
  hs->eos_id = p->eos_token_id;
  hs->threshold = p->confidence_threshold;
  hs->tie_rel = kTieRel;
  hs->sample_t = p->temperature;
  hs->sample_seed = p->seed;
  hs->shift = s->m->cfg.logits_shift ? 1 : 0;
  hs->active_block = -1;
  hs->trace_cap = std::min(p->trace_steps, s->trace_cap);
  if (p->decode_strategy == DRT_STRATEGY_BD3_FIXED_QUOTA) {
    hs->policy = POL_BD3_FIXED_QUOTA;
    hs->exclude_token = -1;
    const int bs = p->block_size;
    int count = 0;
    if (p->max_tokens > 0) {
      const int first = prompt_len / bs;
      const int last = (prompt_len + p->max_tokens - 1) / bs;
      count = last - first + 1;
    }
    const int sched = (p->max_tokens + bs - 1) / bs;
    hs->steps_per_block = sched > 0 ? (p->steps + sched - 1) / sched : 0;
    hs->iteration_limit = count * hs->steps_per_block;
  } else if (pipeline) {
    hs->policy = POL_D2F_PIPELINE;
    hs->iteration_limit = p->steps;
    hs->exclude_token = p->mask_token_id;  // run_decode_loop's exclude_mask_token default
    hs->add_threshold = p->add_threshold;
    hs->activate_threshold = p->activate_threshold;
    hs->pipe_blocks = (p->max_tokens + p->block_size - 1) / p->block_size;
  } else {
    hs->policy = POL_BLOCK_THRESHOLD;
    hs->iteration_limit = p->steps;
    hs->exclude_token = p->mask_token_id;
    hs->rounds_cap = std::max(0, p->rounds_per_block);
  }
  hs->cache_end = prompt_len;
  CK(cudaMemcpyAsync(s->state, hs, sizeof(DecodeState), cudaMemcpyHostToDevice, s->stream));
  // Prefill the prompt (d2f mask with the request's origin).
  CK(cudaEventRecord(s->ev0, s->stream));
  const int64_t launches0 = g_launches;
  TRY(prefill(s, 0, prompt_len, s->origin, p->block_size, 0));
  const int prefill_launches = static_cast<int>(g_launches - launches0);
  CK(cudaEventRecord(s->ev1, s->stream));
  cudaEvent_t e_dec0 = nullptr, e_dec1 = nullptr;
  cudaEvent_t flag_ev[4] = {nullptr, nullptr, nullptr, nullptr};
  CK(cudaEventCreate(&e_dec0));
  CK(cudaEventCreate(&e_dec1));
  for (auto& e : flag_ev) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
  CK(cudaEventRecord(e_dec0, s->stream));
  const int limit = hs->iteration_limit;
  int rc = DRT_OK;
  int replays = 0;
  const auto host0 = std::chrono::steady_clock::now();
  for (int i = 0; i < limit; ++i) {
    ++replays;
    if (cudaGraphLaunch(s->g_step, s->stream) != cudaSuccess) { rc = set_error(DRT_INTERNAL_ERROR, "graph launch failed"); break; }
    cudaMemcpyAsync(&s->hflags[i & 3], &s->state->stopped, sizeof(int), cudaMemcpyDeviceToHost, s->stream);
    cudaEventRecord(flag_ev[i & 3], s->stream);
    if (i >= 2) {
      const int j = (i - 2) & 3;
      if (cudaEventQuery(flag_ev[j]) == cudaSuccess && s->hflags[j]) break;
    }
  }
  const float host_ms = std::chrono::duration<float, std::milli>(std::chrono::steady_clock::now() - host0).count();
  cudaEventRecord(e_dec1, s->stream);
  cudaMemcpyAsync(hs, s->state, sizeof(DecodeState), cudaMemcpyDeviceToHost, s->stream);
  cudaMemcpyAsync(out, s->canvas, sizeof(int) * canvas_len, cudaMemcpyDeviceToHost, s->stream);
  cudaEventRecord(e_total1, s->stream);
  cudaError_t se = cudaStreamSynchronize(s->stream);
  if (rc == DRT_OK && se != cudaSuccess) rc = set_error(DRT_INTERNAL_ERROR, "decode failed: %s", cudaGetErrorString(se));
  float pre_ms = 0.f, dec_ms = 0.f, tot_ms = 0.f;
  cudaEventElapsedTime(&pre_ms, s->ev0, s->ev1);
  cudaEventElapsedTime(&dec_ms, e_dec0, e_dec1);
  cudaEventElapsedTime(&tot_ms, e_total0, e_total1);
  cudaEventDestroy(e_dec0);
  cudaEventDestroy(e_dec1);
  cudaEventDestroy(e_total0);
  cudaEventDestroy(e_total1);
  for (auto& e : flag_ev) cudaEventDestroy(e);
  TRY(rc);
  TRY(check_status(s));
  if (hs->error)
    return set_error(hs->policy == POL_D2F_PIPELINE ? DRT_UNSUPPORTED : DRT_INTERNAL_ERROR,
                     hs->policy == POL_D2F_PIPELINE
                         ? "the d2f_block_pipeline window grew past %d forwarded rows (drive this request through propose_device)"
                         : "device plan rejected the request geometry",
                     kMaxFwdRows);
  if (trace != nullptr && p->trace_steps > 0) {
    const int nt = std::min(hs->forward_count, std::min(p->trace_steps, s->trace_cap));
    static_assert(sizeof(StepTrace) == sizeof(drt_step_trace), "trace layout");
    CK(cudaMemcpy(trace, s->trace, sizeof(StepTrace) * nt, cudaMemcpyDeviceToHost));
  }
  if (result) {
    result->forward_count = hs->forward_count;
    result->iteration_count = hs->iteration_count;
    result->committed_token_count = hs->committed_count;
    result->near_tie_steps = hs->near_tie_steps;
    result->exact_tie_steps = hs->exact_tie_steps;
    result->stopped = hs->stopped;
    result->canvas_len = canvas_len;
    result->prefill_ms = pre_ms;
    result->decode_ms = dec_ms;
    result->total_ms = tot_ms;
    result->kernel_launches = prefill_launches + replays * s->g_step_kernels;
    result->host_enqueue_ms = host_ms;
  }
  s->m_forwards += hs->forward_count;
  s->m_committed += hs->committed_count;
  s->m_near += hs->near_tie_steps;
  s->m_exact += hs->exact_tie_steps;
  s->m_ms += pre_ms + dec_ms;
  s->started = false;
  return DRT_OK;
}

extern "C" int drt_session_tp_handle(drt_session* s, void* handle) {
  REQUIRE(s && handle, "null argument");
  REQUIRE(s->tp_buf != nullptr, "the session's model is not tensor-parallel");
  CK(cudaSetDevice(s->device));
  cudaIpcMemHandle_t h;
  CK(cudaIpcGetMemHandle(&h, s->tp_buf));
  static_assert(sizeof(h) == DRT_TP_HANDLE_BYTES, "IPC handle size");
  memcpy(handle, &h, sizeof(h));
  return DRT_OK;
}

extern "C" int drt_session_tp_connect(drt_session* s, const void* handles, int32_t world) {
  REQUIRE(s && handles, "null argument");
  REQUIRE(s->tp_buf != nullptr, "the session's model is not tensor-parallel");
  REQUIRE(world == s->m->shard.world, "group of %d ranks, model sharded over %d", world, s->m->shard.world);
  REQUIRE(!s->tp_p2p, "session already connected");
  REQUIRE(2 * static_cast<unsigned long long>(s->m->L) < kTpTagSpan, "%d layers exceed the peer-flag tag span", s->m->L);
  CK(cudaSetDevice(s->device));
  const int me = s->m->shard.rank;
  for (int r = 0; r < world; ++r) {
    if (r == me) {
      s->tp_peer[r] = s->tp_buf;
      continue;
    }
    cudaIpcMemHandle_t h;
    memcpy(&h, static_cast<const uint8_t*>(handles) + static_cast<size_t>(r) * DRT_TP_HANDLE_BYTES, sizeof(h));
    void* p = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < r; ++q)
        if (q != me && s->tp_peer[q] != nullptr) cudaIpcCloseMemHandle(s->tp_peer[q]);
      for (int q = 0; q < kTpMaxRanks; ++q) s->tp_peer[q] = nullptr;
      return set_error(DRT_UNSUPPORTED, "peer %d buffer not mappable: %s", r, cudaGetErrorString(e));
    }
    s->tp_peer[r] = static_cast<uint8_t*>(p);
  }
  s->tp_p2p = true;
  // Vocabulary-parallel lm_head: rank r projects the tiles [r T / w, (r + 1) T / w) of the T
  // vocabulary tiles (128 rows each), from its replicated copy of the weight.
  drt_model* m = s->m;
  const int tiles = m->V / 128;
  s->tp_vocab = false;
  if (!m->quantized && m->V % 128 == 0 && tiles >= world) {
    s->lm_t0 = static_cast<int>((static_cast<long long>(me) * tiles) / world);
    s->lm_tiles = static_cast<int>((static_cast<long long>(me + 1) * tiles) / world) - s->lm_t0;
    TRY(map_matrix(&s->m_lm_shard, m->lm_head + static_cast<size_t>(s->lm_t0) * 128 * m->H, s->lm_tiles * 128, m->H, 128));
    s->tp_vocab = true;
  }
  if (s->g_dream) { cudaGraphExecDestroy(s->g_dream); s->g_dream = nullptr; }
  return DRT_OK;
}

extern "C" int drt_session_tp_vocab_parallel(drt_session* s, int32_t enable) {
  REQUIRE(s, "null session");
  REQUIRE(s->tp_p2p, "the session's peers are not mapped (drt_session_tp_connect)");
  REQUIRE(!enable || s->lm_tiles > 0, "this model's lm_head cannot be split by vocabulary over the group");
  if (s->tp_vocab != (enable != 0) && s->g_dream) {
    cudaGraphExecDestroy(s->g_dream);
    s->g_dream = nullptr;
  }
  s->tp_vocab = enable != 0;
  return DRT_OK;
}

namespace {
// A flag pair (flag, epoch) that nothing ever raises: the drill's wait can only run out.
__device__ unsigned long long g_drill_flags[2];

__global__ void peer_wait_drill_kernel(int* status) {
  tp_wait_flags(&g_drill_flags[0], &g_drill_flags[1], 1, 1, status);
}
}  // namespace

extern "C" int drt_session_peer_wait_drill(drt_session* s) {
  REQUIRE(s, "null session");
  CK(cudaSetDevice(s->device));
  CK(launch_k(peer_wait_drill_kernel, dim3(1), dim3(32), 0, s->stream, false, s->status));
  CK(cudaStreamSynchronize(s->stream));
  return check_status(s);
}

extern "C" int drt_entropy_count_schedule(int32_t n_masked, int32_t steps, double eps, int32_t* transfer) {
  REQUIRE(transfer, "null argument");
  REQUIRE(n_masked >= 0 && steps >= 1, "n_masked must be >= 0 and steps >= 1");
  REQUIRE(std::isfinite(eps) && eps >= 0.0 && eps <= 1.0, "eps must be in [0, 1]");
  entropy_count_plan(n_masked, steps, eps, transfer);
  return DRT_OK;
}

extern "C" int drt_session_metrics(drt_session* s, drt_metrics* out) {
  REQUIRE(s && out, "null argument");
  out->forward_count = s->m_forwards;
  out->forwarded_rows = s->m_rows;
  out->prefill_rows = s->m_prefill_rows;
  out->committed_token_count = s->m_committed;
  out->near_tie_steps = s->m_near;
  out->exact_tie_steps = s->m_exact;
  out->forward_ms_total = s->m_ms;
  out->device_bytes = s->bytes;
  return DRT_OK;
}

// ======================================================================= kernel-level entry points
extern "C" size_t drt_selector_scratch_bytes(int32_t n_rows, int32_t vocab) {
  const size_t chunks = (static_cast<size_t>(std::max(vocab, 1)) + kSelChunk - 1) / kSelChunk;
  const size_t np = static_cast<size_t>(std::max(n_rows, 1)) * chunks;
  // chunk partials (max, index, sum; sampled key, runner-up, index), row statistics, counters, and
  // one 256-byte alignment pad per region
  return np * (4 + 4 + 8 + 8 + 8 + 4) + static_cast<size_t>(std::max(n_rows, 1)) * (4 + 8 + 8) + 10 * 256;
}

extern "C" int drt_selector_rows(const float* logits, int64_t ld, int32_t n_rows, int32_t vocab, int32_t mode, double temperature,
                                 void* scratch, double* conf, int32_t* token, void* stream) {
  REQUIRE(logits && scratch && conf && token, "null argument");
  REQUIRE(n_rows >= 0 && vocab >= 1 && ld >= vocab, "bad selector geometry");
  REQUIRE(mode == DRT_SELECT_MAX_PROB || mode == DRT_SELECT_NEG_ENTROPY, "unknown selector mode %d", mode);
  if (n_rows == 0) return DRT_OK;
  REQUIRE(n_rows <= 65535, "at most 65535 rows per call");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int chunks = (vocab + kSelChunk - 1) / kSelChunk;
  const size_t np = static_cast<size_t>(n_rows) * chunks;
  uint8_t* p = static_cast<uint8_t*>(scratch);
  auto take = [&](size_t bytes) { uint8_t* q = p; p += (bytes + 255) & ~size_t(255); return q; };
  SelArgs a;
  memset(&a, 0, sizeof(a));
  a.part_sum = reinterpret_cast<double*>(take(np * 8));
  a.row_amax = reinterpret_cast<double*>(take(static_cast<size_t>(n_rows) * 8));
  a.row_sum = reinterpret_cast<double*>(take(static_cast<size_t>(n_rows) * 8));
  a.part_max = reinterpret_cast<float*>(take(np * 4));
  a.part_idx = reinterpret_cast<int*>(take(np * 4));
  a.counters = reinterpret_cast<int*>(take(static_cast<size_t>(n_rows) * 4));
  if (mode == DRT_SELECT_NEG_ENTROPY) a.part_ent = reinterpret_cast<double*>(take(np * 8));
  CK(cudaMemsetAsync(a.counters, 0, sizeof(int) * n_rows, st));
  a.logits = logits;
  a.ld = ld;
  a.rows = n_rows;
  a.vocab = vocab;
  a.chunk = kSelChunk;
  a.nchunks = chunks;
  a.mode = mode;
  a.temperature = mode == DRT_SELECT_NEG_ENTROPY ? temperature : 0.0;
  a.exclude = -1;
  a.conf = conf;
  a.token = token;
  if (mode == DRT_SELECT_NEG_ENTROPY) {
    CK(launch_k(sel_pass1_kernel<false, true>, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
    CK(launch_k(sel_entropy_kernel, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
  } else {
    CK(launch_k(sel_pass1_kernel<false>, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
  }
  return DRT_OK;
}

extern "C" int drt_selector_gather(const float* logits, int64_t ld, const int32_t* row_index, int32_t n_rows, int32_t vocab,
                                   int32_t mode, double temperature, void* scratch, double* conf, int32_t* token, void* stream) {
  REQUIRE(logits && row_index && scratch && conf && token, "null argument");
  REQUIRE(n_rows >= 0 && vocab >= 1 && ld >= vocab, "bad selector geometry");
  REQUIRE(mode == DRT_SELECT_MAX_PROB || mode == DRT_SELECT_NEG_ENTROPY, "unknown selector mode %d", mode);
  if (n_rows == 0) return DRT_OK;
  REQUIRE(n_rows <= 65535, "at most 65535 rows per call");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int chunks = (vocab + kSelChunk - 1) / kSelChunk;
  const size_t np = static_cast<size_t>(n_rows) * chunks;
  uint8_t* p = static_cast<uint8_t*>(scratch);
  auto take = [&](size_t bytes) { uint8_t* q = p; p += (bytes + 255) & ~size_t(255); return q; };
  SelArgs a;
  memset(&a, 0, sizeof(a));
  a.part_sum = reinterpret_cast<double*>(take(np * 8));
  a.row_amax = reinterpret_cast<double*>(take(static_cast<size_t>(n_rows) * 8));
  a.row_sum = reinterpret_cast<double*>(take(static_cast<size_t>(n_rows) * 8));
  a.part_max = reinterpret_cast<float*>(take(np * 4));
  a.part_idx = reinterpret_cast<int*>(take(np * 4));
  a.counters = reinterpret_cast<int*>(take(static_cast<size_t>(n_rows) * 4));
  if (mode == DRT_SELECT_NEG_ENTROPY) a.part_ent = reinterpret_cast<double*>(take(np * 8));
  CK(cudaMemsetAsync(a.counters, 0, sizeof(int) * n_rows, st));
  a.logits = logits;
  a.ld = ld;
  a.row_index = row_index;
  a.rows = n_rows;
  a.vocab = vocab;
  a.chunk = kSelChunk;
  a.nchunks = chunks;
  a.mode = mode;
  a.temperature = mode == DRT_SELECT_NEG_ENTROPY ? temperature : 0.0;
  a.exclude = -1;
  a.conf = conf;
  a.token = token;
  if (mode == DRT_SELECT_NEG_ENTROPY) {
    CK(launch_k(sel_pass1_kernel<false, true>, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
    CK(launch_k(sel_entropy_kernel, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
  } else {
    CK(launch_k(sel_pass1_kernel<false>, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
  }
  return DRT_OK;
}

extern "C" int drt_selector_sample(const float* logits, int64_t ld, const int32_t* row_index, int32_t n_rows, int32_t vocab,
                                   double temperature, uint64_t seed, int32_t forward, const int32_t* positions,
                                   void* scratch, double* conf, int32_t* token, int32_t* tie, void* stream) {
  REQUIRE(logits && positions && scratch && conf && token, "null argument");
  REQUIRE(n_rows >= 0 && vocab >= 1 && ld >= vocab, "bad selector geometry");
  REQUIRE(std::isfinite(temperature) && temperature > 0.0, "sampling needs a finite temperature > 0");
  REQUIRE(forward >= 0, "forward index must be >= 0");
  if (n_rows == 0) return DRT_OK;
  REQUIRE(n_rows <= 65535, "at most 65535 rows per call");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int chunks = (vocab + kSelChunk - 1) / kSelChunk;
  const size_t np = static_cast<size_t>(n_rows) * chunks;
  uint8_t* p = static_cast<uint8_t*>(scratch);
  auto take = [&](size_t bytes) { uint8_t* q = p; p += (bytes + 255) & ~size_t(255); return q; };
  SelArgs a;
  memset(&a, 0, sizeof(a));
  a.part_sum = reinterpret_cast<double*>(take(np * 8));
  a.part_skey = reinterpret_cast<double*>(take(np * 8));
  a.part_skey2 = reinterpret_cast<double*>(take(np * 8));
  a.row_amax = reinterpret_cast<double*>(take(static_cast<size_t>(n_rows) * 8));
  a.row_sum = reinterpret_cast<double*>(take(static_cast<size_t>(n_rows) * 8));
  a.part_max = reinterpret_cast<float*>(take(np * 4));
  a.part_idx = reinterpret_cast<int*>(take(np * 4));
  a.part_sidx = reinterpret_cast<int*>(take(np * 4));
  a.counters = reinterpret_cast<int*>(take(static_cast<size_t>(n_rows) * 4));
  CK(cudaMemsetAsync(a.counters, 0, sizeof(int) * n_rows, st));
  a.logits = logits;
  a.ld = ld;
  a.row_index = row_index;
  a.rows = n_rows;
  a.vocab = vocab;
  a.chunk = kSelChunk;
  a.nchunks = chunks;
  a.mode = SEL_SAMPLE;
  a.exclude = -1;
  a.sample_t = temperature;
  a.sample_seed = seed;
  a.sample_forward = forward;
  a.positions = positions;
  a.row_tie = tie;
  a.conf = conf;
  a.token = token;
  CK(launch_k(sel_pass1_kernel<true>, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
  return DRT_OK;
}

extern "C" int drt_select_choices(const double* conf, const int32_t* offsets, int32_t n_items, int32_t mode, int32_t k,
                                  double tau, double tie_rel, int32_t* chosen, int32_t* tie, void* stream) {
  REQUIRE(conf && offsets && chosen && tie, "null argument");
  REQUIRE(n_items >= 0 && n_items <= 65535, "n_items outside [0, 65535]");
  REQUIRE(mode == CHOICE_TOPK || mode == CHOICE_THRESHOLD, "unknown choice mode %d", mode);
  REQUIRE(mode != CHOICE_TOPK || k >= 0, "k must be >= 0");
  REQUIRE(tie_rel >= 0.0, "tie_rel must be >= 0");
  if (n_items == 0) return DRT_OK;
  CK(launch_k(sel_choose_kernel, dim3(n_items), dim3(32), 0, static_cast<cudaStream_t>(stream), false, conf, offsets, mode, k, tau,
              tie_rel, chosen, tie));
  return DRT_OK;
}

extern "C" int drt_selector_topp(const float* logits, int64_t ld, const int32_t* row_index, int32_t n_rows, int32_t vocab,
                                 double temperature, double top_p, int32_t exclude_token, double tie_rel, double* conf,
                                 int32_t* token, int32_t* tie, void* stream) {
  REQUIRE(logits && conf && token, "null argument");
  REQUIRE(n_rows >= 0 && n_rows <= 65535 * 16, "n_rows outside [0, %d]", 65535 * 16);
  REQUIRE(vocab >= 1 && ld >= vocab, "vocab must be >= 1 and ld >= vocab");
  REQUIRE(std::isfinite(temperature) && std::isfinite(top_p) && top_p > 0.0, "temperature / top_p invalid");
  REQUIRE(tie_rel >= 0.0, "tie_rel must be >= 0");
  REQUIRE(exclude_token >= -1 && exclude_token < vocab, "exclude_token outside the vocabulary");
  if (n_rows == 0) return DRT_OK;
  TRY(configure_kernels());
  ToppArgs t;
  memset(&t, 0, sizeof(t));
  t.logits = logits;
  t.ld = ld;
  t.row_index = row_index;
  t.rows = n_rows;
  t.vocab = vocab;
  t.temperature = temperature;
  t.top_p = top_p;
  t.exclude = exclude_token;
  t.tie_rel = tie_rel;
  t.conf = conf;
  t.token = token;
  t.tie = tie;
  CK(launch_k(sel_topp_entropy_kernel, dim3(n_rows), dim3(kToppThreads), kToppSmemBytes, static_cast<cudaStream_t>(stream), false, t));
  return DRT_OK;
}

namespace {
__global__ void exp_nonpos_kernel(const double* __restrict__ x, double* __restrict__ y, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[i] = exp_nonpos(x[i]);
}
}  // namespace

extern "C" int drt_exp_nonpos(const double* x, double* y, int64_t n, void* stream) {
  REQUIRE(x && y && n >= 0, "null argument");
  if (n == 0) return DRT_OK;
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4096));
  exp_nonpos_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(x, y, n);
  CK(cudaGetLastError());
  return DRT_OK;
}

extern "C" size_t drt_linear_scratch_bytes(int32_t rows, int32_t n, int32_t K, int32_t splits) {
  (void)rows;
  (void)n;
  (void)K;
  (void)splits;
  return 0;  // split-K partials live in the cluster's shared memory
}

extern "C" int drt_linear_bf16(const void* x, const void* w, float* y, int32_t rows, int32_t n, int32_t K, int32_t splits,
                               int32_t round_bf16, void* scratch, void* stream) {
  (void)scratch;
  REQUIRE(x && w && y, "null argument");
  REQUIRE(rows >= 1 && n >= 128 && n % 128 == 0 && K >= 64 && K % 64 == 0, "linear needs n %% 128 == 0 and K %% 64 == 0");
  REQUIRE(splits == 1 || splits == 2 || splits == 4 || splits == 8 || splits == 16, "splits must be 1, 2, 4, 8 or 16");
  REQUIRE(splits <= K / 64, "splits exceed the K blocks");
  TRY(configure_kernels());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  CUtensorMap ma, mb;
  TRY(map_matrix(&ma, w, n, K, 128));
  TRY(map_matrix(&mb, x, rows, K, 64));
  const int tiles_m = n / 128, tiles_n = (rows + 63) / 64;
  const int kb = K / 64;
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.n_out = n;
  a.K = K;
  a.rows = rows;
  a.splits = splits;
  a.kb_per_split = (kb + splits - 1) / splits;
  a.stages = std::max(1, std::min(a.kb_per_split, 8));
  a.epi = round_bf16 ? EPI_STORE_F32 : EPI_STORE_RAW;
  a.out_f32 = y;
  a.ld_out = n;
  CK(launch_kc(gemm_swapab_kernel<64>, dim3(tiles_m, tiles_n, splits), dim3(128), GemmCfg<64>::smem_bytes(a.stages), st,
               false, splits, ma, mb, a));
  return DRT_OK;
}

extern "C" int drt_linear_q4(const void* x, const void* q, const void* scale, const void* bias, float* y, int32_t rows,
                             int32_t n, int32_t K, int32_t splits, void* stream) {
  REQUIRE(x && q && scale && bias && y, "null argument");
  REQUIRE(rows >= 1 && rows <= kDecRows, "rows must be in [1, %d]", kDecRows);
  REQUIRE(n >= 128 && n % 128 == 0 && K >= 64 && K % 64 == 0, "quantized linear needs n %% 128 == 0 and K %% 64 == 0");
  REQUIRE(splits == 1 || splits == 2 || splits == 4 || splits == 8 || splits == 16, "splits must be 1, 2, 4, 8 or 16");
  const int kb = K / 64;
  const int kbps = (kb + splits - 1) / splits;
  REQUIRE(splits <= kb && kbps <= kDecQMaxKb, "K blocks per split must be in [1, %d]", kDecQMaxKb);
  TRY(configure_kernels());
  CUtensorMap mq, mb;
  TRY(map_u8(&mq, q, n, K / 2, 32, 128));
  TRY(map_matrix(&mb, x, rows, K, 64));
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.n_out = n;
  a.K = K;
  a.rows = rows;
  a.splits = splits;
  a.kb_per_split = kbps;
  a.stages = kDecQStages;
  a.epi = EPI_STORE_F32;
  a.out_f32 = y;
  a.ld_out = n;
  a.q_scale = static_cast<const __nv_bfloat16*>(scale);
  a.q_bias = static_cast<const __nv_bfloat16*>(bias);
  a.q_groups = kb;
  DecGemmKernel kern = dec_gemm_kernel(EPI_STORE_F32, splits, 4);
  CK(launch_kc(kern, dim3(n / 128, 1, splits), dim3(128), dec_q_smem_bytes(kbps, 4), static_cast<cudaStream_t>(stream), false,
               splits, mq, mb, a));
  return DRT_OK;
}

extern "C" int drt_linear_q8(const void* x, const void* q, const void* scale, const void* bias, float* y, int32_t rows,
                             int32_t n, int32_t K, int32_t splits, void* stream) {
  REQUIRE(x && q && scale && bias && y, "null argument");
  REQUIRE(rows >= 1 && rows <= kDecRows, "rows must be in [1, %d]", kDecRows);
  REQUIRE(n >= 128 && n % 128 == 0 && K >= 64 && K % 64 == 0, "quantized linear needs n %% 128 == 0 and K %% 64 == 0");
  REQUIRE(splits == 1 || splits == 2 || splits == 4 || splits == 8 || splits == 16, "splits must be 1, 2, 4, 8 or 16");
  const int kb = K / 64;
  const int kbps = (kb + splits - 1) / splits;
  REQUIRE(splits <= kb && kbps <= kDecQMaxKb, "K blocks per split must be in [1, %d]", kDecQMaxKb);
  TRY(configure_kernels());
  CUtensorMap mq, mb;
  TRY(map_u8(&mq, q, n, K, 64, 128));
  TRY(map_matrix(&mb, x, rows, K, 64));
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.n_out = n;
  a.K = K;
  a.rows = rows;
  a.splits = splits;
  a.kb_per_split = kbps;
  a.stages = kDecQStages;
  a.epi = EPI_STORE_F32;
  a.out_f32 = y;
  a.ld_out = n;
  a.q_scale = static_cast<const __nv_bfloat16*>(scale);
  a.q_bias = static_cast<const __nv_bfloat16*>(bias);
  a.q_groups = kb;
  DecGemmKernel kern = dec_gemm_kernel(EPI_STORE_F32, splits, 8);
  CK(launch_kc(kern, dim3(n / 128, 1, splits), dim3(128), dec_q_smem_bytes(kbps, 8), static_cast<cudaStream_t>(stream), false,
               splits, mq, mb, a));
  return DRT_OK;
}

extern "C" int drt_quantize_q8(const void* w, int64_t rows, int32_t K, void* q, void* scale, void* bias, void* stream) {
  REQUIRE(w && q && scale && bias, "null argument");
  REQUIRE(rows >= 1 && K >= 64 && K % 64 == 0, "quantization needs K %% 64 == 0");
  const int64_t total = rows * (K / 64);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 65535));
  quantize_q8_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(w), rows, K, static_cast<uint8_t*>(q), static_cast<__nv_bfloat16*>(scale),
      static_cast<__nv_bfloat16*>(bias));
  CK(cudaGetLastError());
  return DRT_OK;
}

extern "C" int drt_quantize_q4(const void* w, int64_t rows, int32_t K, void* q, void* scale, void* bias, void* stream) {
  REQUIRE(w && q && scale && bias, "null argument");
  REQUIRE(rows >= 1 && K >= 64 && K % 64 == 0, "quantization needs K %% 64 == 0");
  const int64_t total = rows * (K / 64);
  const unsigned blocks = static_cast<unsigned>(std::min<int64_t>((total + 255) / 256, 65535));
  quantize_q4_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __nv_bfloat16*>(w), rows, K, static_cast<uint8_t*>(q), static_cast<__nv_bfloat16*>(scale),
      static_cast<__nv_bfloat16*>(bias));
  CK(cudaGetLastError());
  return DRT_OK;
}

// ======================================================================= selector without allocation
// drt_selector_rows_noalloc: the fused selector with its scratch (chunk partials, row statistics,
// arrival counters) in one file-scope device array instead of caller memory, for callers that may
// not allocate device memory. The array is fixed at kNoAllocScratchBytes (about 0.81 MB) and every
// GPU that loads this library holds one copy until the process exits.
namespace {
constexpr int kNoAllocMaxRows = 1024;
constexpr int kNoAllocMaxVocab = 262144;
constexpr size_t kNoAllocMaxParts = static_cast<size_t>(kNoAllocMaxRows) * (kNoAllocMaxVocab / kSelChunk);
// part_sum f64 + part_max f32 + part_idx i32 + part_ent f64 per (row, chunk); row_amax f64 + row_sum f64 +
// counter i32 per row; seven 256-byte alignment pads.
constexpr size_t kNoAllocScratchBytes = kNoAllocMaxParts * (8 + 4 + 4 + 8) + static_cast<size_t>(kNoAllocMaxRows) * (8 + 8 + 4) + 7 * 256;
static __device__ __align__(256) uint8_t g_selector_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
struct NoAllocEntry {
  unsigned long long ctx_id;  // process-unique id of the CUDA context (cuCtxGetId)
  void* ptr;
};
std::vector<NoAllocEntry> g_noalloc_cache;

// Id of the calling thread's current CUDA context; false when no context is current yet. Context ids
// are unique for the life of the process, so a context created after cudaDeviceReset (or another
// context on the same device) never matches an address cached for an earlier one.
bool current_ctx_id(unsigned long long* id) {
  typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
  typedef CUresult (*CtxGetIdFn)(CUcontext, unsigned long long*);
  static CtxGetCurrentFn get_current = nullptr;
  static CtxGetIdFn get_id = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_current = reinterpret_cast<CtxGetCurrentFn>(p);
    p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuCtxGetId", &p, 12000, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      get_id = reinterpret_cast<CtxGetIdFn>(p);
  });
  if (get_current == nullptr || get_id == nullptr) return false;
  CUcontext ctx = nullptr;
  if (get_current(&ctx) != CUDA_SUCCESS || ctx == nullptr) return false;
  return get_id(ctx, id) == CUDA_SUCCESS;
}

// Device address of g_selector_scratch in the current context. In host code the symbol is only a
// host-side stand-in, so the address is looked up once per context (with its device current) and
// cached under the context's id.
int noalloc_scratch(void** out) {
  unsigned long long id = 0;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (current_ctx_id(&id)) {
    for (const NoAllocEntry& e : g_noalloc_cache)
      if (e.ctx_id == id) {
        *out = e.ptr;
        return DRT_OK;
      }
  }
  void* p = nullptr;
  const cudaError_t e = cudaGetSymbolAddress(&p, g_selector_scratch);
  if (e != cudaSuccess || p == nullptr)
    return set_error(DRT_INTERNAL_ERROR, "cudaGetSymbolAddress(selector scratch) failed: %s", cudaGetErrorString(e));
  // The lookup made the device's primary context current if none was.
  if (!current_ctx_id(&id)) return set_error(DRT_INTERNAL_ERROR, "no current CUDA context after the symbol lookup");
  if (g_noalloc_cache.size() >= 64) g_noalloc_cache.erase(g_noalloc_cache.begin());
  g_noalloc_cache.push_back({id, p});
  *out = p;
  return DRT_OK;
}
}  // namespace

extern "C" int drt_selector_rows_noalloc(const float* logits, int64_t ld, int32_t n_rows, int32_t vocab, int32_t mode,
                                         double temperature, double* conf, int32_t* token, void* stream) {
  REQUIRE(logits && conf && token, "null argument");
  REQUIRE(n_rows >= 0 && vocab >= 1 && ld >= vocab, "bad selector geometry");
  REQUIRE(mode == DRT_SELECT_MAX_PROB || mode == DRT_SELECT_NEG_ENTROPY, "unknown selector mode %d", mode);
  REQUIRE(n_rows <= kNoAllocMaxRows, "drt_selector_rows_noalloc scores at most %d rows per call (got %d); "
          "use drt_selector_rows with caller scratch for more", kNoAllocMaxRows, n_rows);
  REQUIRE(vocab <= kNoAllocMaxVocab, "drt_selector_rows_noalloc scores rows of at most %d logits (got %d); "
          "use drt_selector_rows with caller scratch for more", kNoAllocMaxVocab, vocab);
  if (n_rows == 0) return DRT_OK;
  void* base = nullptr;
  TRY(noalloc_scratch(&base));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int chunks = (vocab + kSelChunk - 1) / kSelChunk;
  const size_t np = static_cast<size_t>(n_rows) * chunks;
  uint8_t* p = static_cast<uint8_t*>(base);
  auto take = [&](size_t bytes) { uint8_t* q = p; p += (bytes + 255) & ~size_t(255); return q; };
  SelArgs a;
  memset(&a, 0, sizeof(a));
  a.part_sum = reinterpret_cast<double*>(take(np * 8));
  a.row_amax = reinterpret_cast<double*>(take(static_cast<size_t>(n_rows) * 8));
  a.row_sum = reinterpret_cast<double*>(take(static_cast<size_t>(n_rows) * 8));
  a.part_max = reinterpret_cast<float*>(take(np * 4));
  a.part_idx = reinterpret_cast<int*>(take(np * 4));
  a.counters = reinterpret_cast<int*>(take(static_cast<size_t>(n_rows) * 4));
  if (mode == DRT_SELECT_NEG_ENTROPY) a.part_ent = reinterpret_cast<double*>(take(np * 8));
  if (static_cast<size_t>(p - static_cast<uint8_t*>(base)) > kNoAllocScratchBytes)
    return set_error(DRT_INTERNAL_ERROR, "selector scratch layout exceeds the static array");
  // The array keeps the previous call's contents; the arrival counters must start at zero.
  CK(cudaMemsetAsync(a.counters, 0, sizeof(int) * n_rows, st));
  a.logits = logits;
  a.ld = ld;
  a.rows = n_rows;
  a.vocab = vocab;
  a.chunk = kSelChunk;
  a.nchunks = chunks;
  a.mode = mode;
  a.temperature = mode == DRT_SELECT_NEG_ENTROPY ? temperature : 0.0;
  a.exclude = -1;
  a.conf = conf;
  a.token = token;
  if (mode == DRT_SELECT_NEG_ENTROPY) {
    CK(launch_k(sel_pass1_kernel<false, true>, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
    CK(launch_k(sel_entropy_kernel, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
  } else {
    CK(launch_k(sel_pass1_kernel<false>, dim3(chunks, n_rows), dim3(kSelThreads), 0, st, false, a));
  }
  return DRT_OK;
}
