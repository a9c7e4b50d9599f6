// Host side of libgemm3_b200.so: argument validation, TMA descriptor encoding and kernel
// launches behind the extern "C" entry points declared in include/nvfp4_gemm.h.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/nvfp4_gemm.h"
#include "gemm_kernel.cuh"
#include "gemm_pair_kernel.cuh"
#include "gemm_stream_kernel.cuh"
#include "quant_kernel.cuh"

namespace {

thread_local int32_t g_last_cuda_error = 0;

int cuda_fail(cudaError_t e) {
  g_last_cuda_error = static_cast<int32_t>(e);
  return NVFP4_ERR_CUDA;
}

#define G3_CUDA(expr)                          \
  do {                                         \
    cudaError_t e_ = (expr);                   \
    if (e_ != cudaSuccess) return cuda_fail(e_); \
  } while (0)

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) & (a - 1)) == 0; }

constexpr int kMaxDevices = 64;

struct DeviceCache {
  bool ready = false;
  int sm_count = 0;
  int cc_major = 0, cc_minor = 0;
  int64_t l2_bytes = 0;
  bool gemm_attr_set = false;
  bool stream_attr_set = false;
  int pair_clusters = 0;  // co-resident CTA pairs of the pair kernel
  // co-resident 256-thread quantiser blocks per SM, per input dtype and QuantKind
  int quant_blocks[3][3] = {{0, 0, 0}, {0, 0, 0}, {0, 0, 0}};
};
DeviceCache g_dev[kMaxDevices];
std::mutex g_mu;
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

int current_device(int* dev) {
  G3_CUDA(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= kMaxDevices) return NVFP4_ERR_INVALID_VALUE;
  return NVFP4_OK;
}

int device_cache(int dev, DeviceCache** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceCache& d = g_dev[dev];
  if (!d.ready) {
    cudaDeviceProp prop;
    G3_CUDA(cudaGetDeviceProperties(&prop, dev));
    d.sm_count = prop.multiProcessorCount;
    d.cc_major = prop.major;
    d.cc_minor = prop.minor;
    d.l2_bytes = prop.l2CacheSize;
    d.ready = true;
  }
  *out = &d;
  return NVFP4_OK;
}

typedef CUresult (*PFN_addr_range)(CUdeviceptr*, size_t*, CUdeviceptr);
PFN_addr_range g_addr_range = nullptr;

int get_address_range() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_addr_range != nullptr) return NVFP4_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  G3_CUDA(cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q));
  if (fn == nullptr || q != cudaDriverEntryPointSuccess) return NVFP4_ERR_UNSUPPORTED;
  g_addr_range = reinterpret_cast<PFN_addr_range>(fn);
  return NVFP4_OK;
}

int get_encoder() {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_encode != nullptr) return NVFP4_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  G3_CUDA(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
  if (fn == nullptr || q != cudaDriverEntryPointSuccess) return NVFP4_ERR_UNSUPPORTED;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return NVFP4_OK;
}

// 2-D uint8 view [rows, row_bytes] of a packed operand, boxes of box_rows x 128 bytes with the
// 128-byte swizzle; reads outside the tensor are zero-filled by TMA.
int encode_operand(CUtensorMap* m, const void* base, int64_t rows, int64_t row_bytes, uint32_t box_rows) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(row_bytes)};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(g3::kTileKBytes), box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NVFP4_OK : NVFP4_ERR_TENSOR_MAP;
}

// Opt the GEMM kernels into their dynamic shared memory once per device (outside any capture).
int ensure_gemm_attributes(DeviceCache* d) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (d->gemm_attr_set) return NVFP4_OK;
  G3_CUDA(cudaFuncSetAttribute(g3::nvfp4_gemm_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               g3::kGemmSmemBytes));
  G3_CUDA(cudaFuncSetAttribute(g3::nvfp4_gemm_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               g3::kGemmSmemBytes));
  G3_CUDA(cudaFuncSetAttribute(g3::nvfp4_gemm_pair_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               g3::kPairSmemBytes));
  G3_CUDA(cudaFuncSetAttribute(g3::nvfp4_gemm_pair_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                               g3::kPairSmemBytes));
  // How many CTA pairs fit at once (SMs that cannot be paired inside a GPC stay idle).
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(2 * (d->sm_count / 2), 1, 1);
  lc.blockDim = dim3(g3::kPairThreads, 1, 1);
  lc.dynamicSmemBytes = g3::kPairSmemBytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = 2;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  lc.attrs = &attr;
  lc.numAttrs = 1;
  int n = 0;
  if (cudaOccupancyMaxActiveClusters(&n, g3::nvfp4_gemm_pair_kernel<true>, &lc) != cudaSuccess || n < 1) {
    (void)cudaGetLastError();
    n = d->sm_count / 2;
  }
  d->pair_clusters = n;
  d->gemm_attr_set = true;
  return NVFP4_OK;
}

// 3-D uint32 view of a swizzled scale tensor: {128 words = one 512-byte chunk, 64-element block,
// 128-row block}; boxes of `box_rb` row blocks x one pair-kernel stage of blocks. Out-of-range
// blocks read as zero.
int encode_scales(CUtensorMap* m, const void* base, int64_t rowblocks, int64_t kblocks, uint32_t box_rb) {
  cuuint64_t dims[3] = {128, static_cast<cuuint64_t>(kblocks), static_cast<cuuint64_t>(rowblocks)};
  cuuint64_t strides[2] = {512, static_cast<cuuint64_t>(kblocks) * 512};
  cuuint32_t box[3] = {128, static_cast<cuuint32_t>(g3::kPairKBlocks), box_rb};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? NVFP4_OK : NVFP4_ERR_TENSOR_MAP;
}

int grid_for(int64_t work, int sm_count, int threads = 256) {
  const int64_t want = (work + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(sm_count) * 8;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

// The quantiser kernels: one block per thread with 32-bit indices whenever every element offset
// of the padded scale grid (rows_pad x k) fits in 32 bits, else with 64-bit ones; and, for 16-bit
// inputs whose rows hold whole pairs of blocks and whose outputs are aligned for the wider
// stores, two blocks per thread.
enum QuantKind { kQuantIdx32 = 0, kQuantIdx64 = 1, kQuantPair = 2 };

bool quant_idx32(const g3::QuantParams& p) { return p.rows_pad * p.k < (int64_t(1) << 32); }

QuantKind quant_kind(const g3::QuantParams& p, int32_t in_dtype) {
  if (!quant_idx32(p)) return kQuantIdx64;
  if (in_dtype != NVFP4_DTYPE_F32 && p.k % 32 == 0 && aligned(p.packed, 16) && aligned(p.sf_swz, 2) &&
      (p.sf_lin == nullptr || aligned(p.sf_lin, 2)))
    return kQuantPair;
  return kQuantIdx32;
}

template <int kInDtype>
void* quant_kernel_fn(QuantKind kind) {
  switch (kind) {
    case kQuantIdx32: return reinterpret_cast<void*>(g3::nvfp4_quantize_kernel<kInDtype, uint32_t>);
    case kQuantIdx64: return reinterpret_cast<void*>(g3::nvfp4_quantize_kernel<kInDtype, int64_t>);
    default:
      if constexpr (kInDtype != 2) return reinterpret_cast<void*>(g3::nvfp4_quantize_pair_kernel<kInDtype>);
      return nullptr;  // not selected for f32 (quant_kind)
  }
}

void* quant_kernel_for(int32_t in_dtype, QuantKind kind) {
  switch (in_dtype) {
    case NVFP4_DTYPE_F16: return quant_kernel_fn<0>(kind);
    case NVFP4_DTYPE_BF16: return quant_kernel_fn<1>(kind);
    default: return quant_kernel_fn<2>(kind);
  }
}

// One full wave of the grid-stride quantiser: every SM holds as many blocks as fit, so no
// partial second wave is left at the end.
int quant_grid(DeviceCache* d, int32_t in_dtype, QuantKind kind, int64_t work) {
  int& per_sm = d->quant_blocks[in_dtype][kind];
  if (per_sm == 0) {
    std::lock_guard<std::mutex> lock(g_mu);
    int n = 0;
    const cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, quant_kernel_for(in_dtype, kind), 256, 0);
    if (e != cudaSuccess || n < 1) {
      (void)cudaGetLastError();
      n = 4;
    }
    per_sm = n;
  }
  const int64_t want = (work + 255) / 256;
  const int64_t cap = static_cast<int64_t>(d->sm_count) * per_sm;
  return static_cast<int>(want < 1 ? 1 : (want > cap ? cap : want));
}

// A bounded wait that can never complete: one thread waits on a fresh mbarrier (count 1) that
// nothing arrives at, through the same mbar_wait the GEMM kernels use. After kWaitTimeoutNs it
// records `code` in *status and returns; the kernel then exits normally.
__global__ void wait_timeout_selftest_kernel(int* status, int code) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    g3::mbar_init(&bar, 1);
    g3::fence_mbarrier_init();
    if (g3::mbar_wait(&bar, 0, status, code, nullptr)) atomicExch(status, -1);  // cannot happen
  }
}

// Where the epilogue writes C: a row-major view with row stride ldc starting at column col0 of
// `c`, and optionally the same view in other GPUs' buffers (the fused gather).
struct OutputSpec {
  void* c = nullptr;
  int64_t ldc = 0, col0 = 0;
  int n_peer = 0;
  void* peer[g3::kMaxPeers] = {};
};

template <typename P>
void set_output(P& p, const OutputSpec& o) {
  p.c = o.c;
  p.ldc = o.ldc;
  p.col0 = o.col0;
  p.n_peer = o.n_peer;
  for (int d = 0; d < g3::kMaxPeers; ++d) p.peer[d] = d < o.n_peer ? o.peer[d] : nullptr;
}

// Weight-streaming kernel (gemm_stream_kernel.cuh) for M <= 128: B in 128-row tiles over a
// persistent grid of at most one CTA per SM, all of A in the MMA's N dimension.
int launch_stream(const void* a, const void* b, const void* sfa, const void* sfb, const OutputSpec& out,
                  const float* alpha, int64_t m, int64_t n, int64_t k, int32_t out_dtype, const nvfp4_gemm_config& def,
                  int32_t* status, void* stream) {
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  DeviceCache* d = nullptr;
  rc = device_cache(dev, &d);
  if (rc != NVFP4_OK) return rc;
  if (d->cc_major != 10) return NVFP4_ERR_UNSUPPORTED;
  rc = get_encoder();
  if (rc != NVFP4_OK) return rc;
  const int n_mma = static_cast<int>((m + 15) / 16 * 16);
  const int a_box_rows = static_cast<int>((m + 7) / 8 * 8);
  CUtensorMap tmap_a, tmap_b;
  rc = encode_operand(&tmap_a, a, m, k / 2, static_cast<uint32_t>(a_box_rows));
  if (rc != NVFP4_OK) return rc;
  rc = encode_operand(&tmap_b, b, n, k / 2, g3::kStreamTileN);
  if (rc != NVFP4_OK) return rc;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    if (!d->stream_attr_set) {
      G3_CUDA(cudaFuncSetAttribute(g3::nvfp4_gemm_stream_kernel<true, false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kStreamSmemLimit));
      G3_CUDA(cudaFuncSetAttribute(g3::nvfp4_gemm_stream_kernel<false, false>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kStreamSmemLimit));
      G3_CUDA(cudaFuncSetAttribute(g3::nvfp4_gemm_stream_kernel<true, true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kStreamSmemLimit));
      G3_CUDA(cudaFuncSetAttribute(g3::nvfp4_gemm_stream_kernel<false, true>,
                                   cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kStreamSmemLimit));
      d->stream_attr_set = true;
    }
  }
  g3::StreamParams p;
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.sfb = static_cast<const uint8_t*>(sfb);
  set_output(p, out);
  p.alpha = alpha;
  p.status = status;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.n_mma = n_mma;
  p.a_box_rows = a_box_rows;
  p.sf_kblocks = static_cast<int>(k / 64);
  p.k_iters = (p.sf_kblocks + g3::kStreamKBlocks - 1) / g3::kStreamKBlocks;
  p.num_tiles = static_cast<int>((n + g3::kStreamTileN - 1) / g3::kStreamTileN);
  p.stages = g3::stream_stages(n_mma);
  p.stage_bytes = g3::stream_stage_bytes(n_mma);
  p.pdl = def.pdl;
  p.pol_b = def.l2_policy_b;
  p.pol_sfb = def.l2_policy_sfb;
  int ctas = d->sm_count;
  if (def.max_ctas > 0 && def.max_ctas < ctas) ctas = def.max_ctas;
  if (ctas > p.num_tiles) ctas = p.num_tiles;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(ctas, 1, 1);
  lc.blockDim = dim3(g3::kStreamThreads, 1, 1);
  lc.dynamicSmemBytes = g3::stream_smem_bytes(n_mma);
  lc.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = &attr;
  lc.numAttrs = def.pdl != 0 ? 1 : 0;
  const bool view = out.n_peer > 0 || out.ldc != n || out.col0 != 0;
  if (out_dtype == NVFP4_DTYPE_BF16)
    G3_CUDA(view ? cudaLaunchKernelEx(&lc, g3::nvfp4_gemm_stream_kernel<true, true>, tmap_a, tmap_b, p)
                 : cudaLaunchKernelEx(&lc, g3::nvfp4_gemm_stream_kernel<true, false>, tmap_a, tmap_b, p));
  else
    G3_CUDA(view ? cudaLaunchKernelEx(&lc, g3::nvfp4_gemm_stream_kernel<false, true>, tmap_a, tmap_b, p)
                 : cudaLaunchKernelEx(&lc, g3::nvfp4_gemm_stream_kernel<false, false>, tmap_a, tmap_b, p));
  return NVFP4_OK;
}

}  // namespace

extern "C" {

int32_t nvfp4_abi_version(void) { return 1; }

int nvfp4_selftest_wait_timeout(int32_t* status, int32_t code, void* stream) {
  if (status == nullptr || code < NVFP4_DEV_TIMEOUT_FULL || code > NVFP4_DEV_ABORTED) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned(status, 4)) return NVFP4_ERR_MISALIGNED;
  wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(reinterpret_cast<int*>(status), code);
  G3_CUDA(cudaGetLastError());
  return NVFP4_OK;
}

int32_t nvfp4_last_cuda_error(void) { return g_last_cuda_error; }

const char* nvfp4_strerror(int32_t code) {
  switch (code) {
    case NVFP4_OK: return "success";
    case NVFP4_ERR_INVALID_VALUE: return "invalid value (shape, pointer or dtype)";
    case NVFP4_ERR_MISALIGNED: return "misaligned pointer";
    case NVFP4_ERR_UNSUPPORTED: return "unsupported device or feature (needs sm_100)";
    case NVFP4_ERR_CUDA: return "CUDA runtime error";
    case NVFP4_ERR_TENSOR_MAP: return "cuTensorMapEncodeTiled rejected the operand";
    case NVFP4_ERR_TOO_LARGE: return "input larger than NVFP4_NOALLOC_MAX_ELEMENTS (2^31 elements)";
    case NVFP4_DEV_TIMEOUT_FULL: return "device timeout: MMA issuer waiting for a filled stage";
    case NVFP4_DEV_TIMEOUT_EMPTY: return "device timeout: producer waiting for a free stage";
    case NVFP4_DEV_TIMEOUT_ACC_FULL: return "device timeout: epilogue waiting for the accumulator";
    case NVFP4_DEV_TIMEOUT_ACC_EMPTY: return "device timeout: MMA issuer waiting for the epilogue";
    case NVFP4_DEV_TIMEOUT_DRAIN: return "device timeout: draining in-flight copies";
    case NVFP4_DEV_ABORTED: return "device abort";
    default: return "unknown status";
  }
}

int nvfp4_device_info(int32_t device, int32_t* sm_count, int32_t* cc_major, int32_t* cc_minor, int64_t* l2_bytes) {
  if (device < 0 || device >= kMaxDevices) return NVFP4_ERR_INVALID_VALUE;
  DeviceCache* d = nullptr;
  int rc = device_cache(device, &d);
  if (rc != NVFP4_OK) return rc;
  if (sm_count) *sm_count = d->sm_count;
  if (cc_major) *cc_major = d->cc_major;
  if (cc_minor) *cc_minor = d->cc_minor;
  if (l2_bytes) *l2_bytes = d->l2_bytes;
  return NVFP4_OK;
}

int nvfp4_set_persisting_l2(int64_t bytes, int64_t* old_bytes) {
  if (bytes < 0) return NVFP4_ERR_INVALID_VALUE;
  size_t old = 0;
  G3_CUDA(cudaDeviceGetLimit(&old, cudaLimitPersistingL2CacheSize));
  G3_CUDA(cudaDeviceSetLimit(cudaLimitPersistingL2CacheSize, static_cast<size_t>(bytes)));
  if (old_bytes) *old_bytes = static_cast<int64_t>(old);
  return NVFP4_OK;
}

int nvfp4_max_active_clusters(int32_t cluster_size, int32_t* out) {
  if (out == nullptr || cluster_size < 1) return NVFP4_ERR_INVALID_VALUE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  DeviceCache* d = nullptr;
  rc = device_cache(dev, &d);
  if (rc != NVFP4_OK) return rc;
  if (d->cc_major != 10) return NVFP4_ERR_UNSUPPORTED;
  // The kernel gemm() launches by default (tile 256x256): the CTA-pair kernel, with its thread
  // count and shared memory; its own launches use clusters of 2.
  auto kern = g3::nvfp4_gemm_pair_kernel<true>;
  G3_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, g3::kPairSmemBytes));
  if (cluster_size > 8) G3_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster_size * d->sm_count, 1, 1);
  cfg.blockDim = dim3(g3::kPairThreads, 1, 1);
  cfg.dynamicSmemBytes = g3::kPairSmemBytes;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeClusterDimension;
  attr.val.clusterDim.x = cluster_size;
  attr.val.clusterDim.y = 1;
  attr.val.clusterDim.z = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = 1;
  int n = 0;
  cudaError_t e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
  if (e != cudaSuccess) {
    (void)cudaGetLastError();
    n = d->sm_count / cluster_size;  // same fallback as nvfp4_gemm_cute/hw.py:20-22
  }
  *out = n;
  return NVFP4_OK;
}

static int gemm_run_impl(const void* a, const void* b, const void* sfa, const void* sfb, const OutputSpec& out,
                         const float* alpha, int64_t m, int64_t n, int64_t k, int32_t out_dtype,
                         const nvfp4_gemm_config* cfg, int32_t* status, void* stream) {
  if (!a || !b || !sfa || !sfb || !out.c || !alpha) return NVFP4_ERR_INVALID_VALUE;
  if (m < 1 || n < 64 || k < 64 || n % 64 || k % 64) return NVFP4_ERR_INVALID_VALUE;
  if (m > INT32_MAX / 2 || n > INT32_MAX / 2 || k > INT32_MAX / 2) return NVFP4_ERR_INVALID_VALUE;
  if (out_dtype != NVFP4_DTYPE_F16 && out_dtype != NVFP4_DTYPE_BF16) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned(a, 16) || !aligned(b, 16) || !aligned(sfa, 16) || !aligned(sfb, 16) || !aligned(out.c, 32) ||
      !aligned(alpha, 4))
    return NVFP4_ERR_MISALIGNED;
  nvfp4_gemm_config def = {};
  if (cfg != nullptr && cfg->struct_size > 0) {
    // The first struct_size bytes: fields added after the caller's version keep their defaults.
    const size_t nbytes = static_cast<size_t>(cfg->struct_size) < sizeof(def) ? static_cast<size_t>(cfg->struct_size)
                                                                             : sizeof(def);
    std::memcpy(&def, cfg, nbytes);
  }
  if ((def.tile_m != 0 && def.tile_m != 128 && def.tile_m != 256) ||
      (def.tile_n != 0 && def.tile_n != 256 && def.tile_n != 128))
    return NVFP4_ERR_INVALID_VALUE;
  if (def.pdl < 0 || def.pdl > 2) return NVFP4_ERR_INVALID_VALUE;
  if (def.tile_n == 128) {
    if (def.tile_m != 128 || m > g3::kStreamMaxM) return NVFP4_ERR_INVALID_VALUE;
    return launch_stream(a, b, sfa, sfb, out, alpha, m, n, k, out_dtype, def, status, stream);
  }
  const bool pair = def.tile_m != 128;
  if (def.raster_band < 0) return NVFP4_ERR_INVALID_VALUE;

  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  DeviceCache* d = nullptr;
  rc = device_cache(dev, &d);
  if (rc != NVFP4_OK) return rc;
  if (d->cc_major != 10) return NVFP4_ERR_UNSUPPORTED;
  rc = get_encoder();
  if (rc != NVFP4_OK) return rc;

  CUtensorMap tmap_a, tmap_b, tmap_sfa, tmap_sfb;
  // A box rows: 128, or for the one-CTA kernel with M < 128 just the rows that exist (rounded
  // up to 8, the swizzle atom).
  const int64_t a_box_rows = (!pair && m < g3::kTileM) ? (m + 7) / 8 * 8 : g3::kTileM;
  rc = encode_operand(&tmap_a, a, m, k / 2, static_cast<uint32_t>(a_box_rows));
  if (rc != NVFP4_OK) return rc;
  rc = encode_operand(&tmap_b, b, n, k / 2, pair ? 128 : g3::kTileN);
  if (rc != NVFP4_OK) return rc;
  if (pair) {
    rc = encode_scales(&tmap_sfa, sfa, (m + 127) / 128, k / 64, 1);
    if (rc != NVFP4_OK) return rc;
    rc = encode_scales(&tmap_sfb, sfb, (n + 127) / 128, k / 64, 2);
    if (rc != NVFP4_OK) return rc;
  }

  g3::GemmParams p;
  p.sfa = static_cast<const uint8_t*>(sfa);
  p.sfb = static_cast<const uint8_t*>(sfb);
  set_output(p, out);
  p.alpha = alpha;
  p.status = status;
  p.m = static_cast<int>(m);
  p.n = static_cast<int>(n);
  p.k = static_cast<int>(k);
  const int tile_rows = pair ? g3::kPairTileM : g3::kTileM;
  p.m_tiles = static_cast<int>((m + tile_rows - 1) / tile_rows);
  p.n_tiles = static_cast<int>((n + g3::kTileN - 1) / g3::kTileN);
  p.k_tiles = static_cast<int>((k + 255) / 256);
  p.sf_kblocks = static_cast<int>(k / 64);
  p.a_box_bytes = static_cast<int>(a_box_rows) * g3::kTileKBytes;
  p.n_rowblocks = static_cast<int>((n + 127) / 128);
  const int64_t tiles = static_cast<int64_t>(p.m_tiles) * p.n_tiles;
  if (tiles > INT32_MAX) return NVFP4_ERR_INVALID_VALUE;
  p.num_tiles = static_cast<int>(tiles);
  // raster_band counts 128-row tiles; the pair kernel's tiles are 256 rows
  p.raster_band = pair ? (def.raster_band + 1) / 2 : def.raster_band;
  p.raster_along_m = def.raster_along_m;
  p.pol_a = def.l2_policy_a;
  p.pol_b = def.l2_policy_b;
  p.pol_sfa = def.l2_policy_sfa;
  p.pol_sfb = def.l2_policy_sfb;
  p.store_evict_first = def.store_evict_first == 0 ? (k >= 8192) : (def.store_evict_first == 1);
  if (out.n_peer > 0) p.store_evict_first = 0;  // the rows are read back at once for the peers
  p.pace_ns = def.epi_store_pace_ns;
  p.tma_b_first = def.tma_b_first;

  rc = ensure_gemm_attributes(d);
  if (rc != NVFP4_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // With cfg->pdl != 0 both kernels launch with programmatic stream serialisation: they wait for
  // the preceding kernel on the device (griddepcontrol.wait) instead of at launch. They read
  // and write nothing global before that wait, so modes 1 and 2 act the same here.
  cudaLaunchAttribute attrs[2];
  int n_attrs = 0;
  if (def.pdl != 0) {
    attrs[n_attrs].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[n_attrs].val.programmaticStreamSerializationAllowed = 1;
    ++n_attrs;
  }
  cudaLaunchConfig_t lc = {};
  lc.stream = s;
  lc.attrs = attrs;
  if (pair) {
    int pairs = d->pair_clusters;
    if (def.max_ctas > 0 && def.max_ctas / 2 < pairs) pairs = def.max_ctas / 2 > 0 ? def.max_ctas / 2 : 1;
    if (pairs > p.num_tiles) pairs = p.num_tiles;
    lc.gridDim = dim3(2 * pairs, 1, 1);
    lc.blockDim = dim3(g3::kPairThreads, 1, 1);
    lc.dynamicSmemBytes = g3::kPairSmemBytes;
    attrs[n_attrs].id = cudaLaunchAttributeClusterDimension;
    attrs[n_attrs].val.clusterDim.x = 2;
    attrs[n_attrs].val.clusterDim.y = 1;
    attrs[n_attrs].val.clusterDim.z = 1;
    lc.numAttrs = n_attrs + 1;
    if (out_dtype == NVFP4_DTYPE_BF16)
      G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_gemm_pair_kernel<true>, tmap_a, tmap_b, tmap_sfa, tmap_sfb, p));
    else
      G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_gemm_pair_kernel<false>, tmap_a, tmap_b, tmap_sfa, tmap_sfb, p));
  } else {
    int ctas = d->sm_count;
    if (def.max_ctas > 0 && def.max_ctas < ctas) ctas = def.max_ctas;
    if (ctas > p.num_tiles) ctas = p.num_tiles;
    lc.gridDim = dim3(ctas, 1, 1);
    lc.blockDim = dim3(g3::kGemmThreads, 1, 1);
    lc.dynamicSmemBytes = g3::kGemmSmemBytes;
    lc.numAttrs = n_attrs;
    if (out_dtype == NVFP4_DTYPE_BF16)
      G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_gemm_kernel<true>, tmap_a, tmap_b, p));
    else
      G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_gemm_kernel<false>, tmap_a, tmap_b, p));
  }
  G3_CUDA(cudaGetLastError());
  return NVFP4_OK;
}

int nvfp4_gemm_run(const void* a, const void* b, const void* sfa, const void* sfb, void* c, const float* alpha,
                   int64_t m, int64_t n, int64_t k, int32_t out_dtype, const nvfp4_gemm_config* cfg, int32_t* status,
                   void* stream) {
  OutputSpec o;
  o.c = c;
  o.ldc = n;
  return gemm_run_impl(a, b, sfa, sfb, o, alpha, m, n, k, out_dtype, cfg, status, stream);
}

int nvfp4_gemm_run_gather(const void* a, const void* b, const void* sfa, const void* sfb, void* const* c_dst,
                          int32_t n_dst, int64_t ldc, int64_t col0, const float* alpha, int64_t m, int64_t n, int64_t k,
                          int32_t out_dtype, const nvfp4_gemm_config* cfg, int32_t* status, void* stream) {
  if (c_dst == nullptr || n_dst < 1 || n_dst > NVFP4_MAX_GATHER_DST) return NVFP4_ERR_INVALID_VALUE;
  if (col0 < 0 || ldc < col0 + n || ldc % 16 || col0 % 16) return NVFP4_ERR_INVALID_VALUE;
  OutputSpec o;
  o.c = c_dst[0];
  o.ldc = ldc;
  o.col0 = col0;
  o.n_peer = n_dst - 1;
  for (int d = 1; d < n_dst; ++d) {
    if (c_dst[d] == nullptr) return NVFP4_ERR_INVALID_VALUE;
    if (!aligned(c_dst[d], 16)) return NVFP4_ERR_MISALIGNED;
    o.peer[d - 1] = c_dst[d];
  }
  return gemm_run_impl(a, b, sfa, sfb, o, alpha, m, n, k, out_dtype, cfg, status, stream);
}

int nvfp4_ipc_get_handle(const void* ptr, void* handle, int64_t* offset) {
  if (ptr == nullptr || handle == nullptr || offset == nullptr) return NVFP4_ERR_INVALID_VALUE;
  int rc = get_address_range();
  if (rc != NVFP4_OK) return rc;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (g_addr_range(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return NVFP4_ERR_INVALID_VALUE;
  cudaIpcMemHandle_t h;
  G3_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  static_assert(sizeof(cudaIpcMemHandle_t) == NVFP4_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return NVFP4_OK;
}

int nvfp4_ipc_open(const void* handle, int64_t offset, void** ptr) {
  if (handle == nullptr || ptr == nullptr || offset < 0) return NVFP4_ERR_INVALID_VALUE;
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  G3_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *ptr = static_cast<uint8_t*>(base) + offset;
  return NVFP4_OK;
}

int nvfp4_ipc_close(void* ptr, int64_t offset) {
  if (ptr == nullptr || offset < 0) return NVFP4_ERR_INVALID_VALUE;
  G3_CUDA(cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset));
  return NVFP4_OK;
}

int nvfp4_quantize(const void* x, int32_t in_dtype, int64_t rows, int64_t k, float global_scale, const float* gs_dev,
                   int32_t gs_mode, int32_t div_mode, void* packed, void* sf_swizzled, void* sf_linear, float* gs_out,
                   void* stream) {
  if (!x || !packed || !sf_swizzled) return NVFP4_ERR_INVALID_VALUE;
  if (rows < 1 || k < 16 || k % 16) return NVFP4_ERR_INVALID_VALUE;
  if (in_dtype < NVFP4_DTYPE_F16 || in_dtype > NVFP4_DTYPE_F32) return NVFP4_ERR_INVALID_VALUE;
  if (gs_mode < 0 || gs_mode > 2 || (gs_mode != 0 && gs_dev == nullptr)) return NVFP4_ERR_INVALID_VALUE;
  if (div_mode != 0 && div_mode != 1) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned(x, 16) || !aligned(packed, 8)) return NVFP4_ERR_MISALIGNED;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  DeviceCache* d = nullptr;
  rc = device_cache(dev, &d);
  if (rc != NVFP4_OK) return rc;
  g3::QuantParams p;
  p.x = x;
  p.rows = rows;
  p.k = k;
  p.cols = k / 16;
  p.rows_pad = (rows + 127) / 128 * 128;
  p.cols_pad = (p.cols + 3) / 4 * 4;
  p.gs = global_scale;
  p.gs_dev = gs_dev;
  p.gs_mode = gs_mode;
  p.div_mode = div_mode;
  p.packed = static_cast<uint8_t*>(packed);
  p.sf_swz = static_cast<uint8_t*>(sf_swizzled);
  p.sf_lin = static_cast<uint8_t*>(sf_linear);
  p.gs_out = gs_out;
  const QuantKind kind = quant_kind(p, in_dtype);
  const int64_t work = kind == kQuantPair ? p.rows_pad * (p.cols_pad / 2) : p.rows_pad * p.cols_pad;
  const int grid = quant_grid(d, in_dtype, kind, work);
  void* args[] = {&p};
  G3_CUDA(cudaLaunchKernel(quant_kernel_for(in_dtype, kind), dim3(static_cast<unsigned>(grid)), dim3(256), args, 0,
                           static_cast<cudaStream_t>(stream)));
  return NVFP4_OK;
}

int nvfp4_amax(const void* x, int32_t in_dtype, int64_t numel, float* amax_out, void* stream) {
  if (!x || !amax_out || numel < 1) return NVFP4_ERR_INVALID_VALUE;
  if (in_dtype < NVFP4_DTYPE_F16 || in_dtype > NVFP4_DTYPE_F32) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned(x, 16) || !aligned(amax_out, 4)) return NVFP4_ERR_MISALIGNED;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  DeviceCache* d = nullptr;
  rc = device_cache(dev, &d);
  if (rc != NVFP4_OK) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  G3_CUDA(cudaMemsetAsync(amax_out, 0, sizeof(float), s));
  const int64_t nvec = numel / 16;
  int grid = grid_for(nvec > 0 ? nvec : 1, d->sm_count);
  const int64_t tail = numel - nvec * 16;
  if (static_cast<int64_t>(grid) * 256 < tail) grid = static_cast<int>((tail + 255) / 256);
  unsigned int* bits = reinterpret_cast<unsigned int*>(amax_out);
  switch (in_dtype) {
    case NVFP4_DTYPE_F16: g3::nvfp4_amax_kernel<0><<<grid, 256, 0, s>>>(x, numel, bits); break;
    case NVFP4_DTYPE_BF16: g3::nvfp4_amax_kernel<1><<<grid, 256, 0, s>>>(x, numel, bits); break;
    default: g3::nvfp4_amax_kernel<2><<<grid, 256, 0, s>>>(x, numel, bits); break;
  }
  G3_CUDA(cudaGetLastError());
  return NVFP4_OK;
}

int nvfp4_quantize_act(const void* x, int32_t in_dtype, int64_t rows, int64_t k, const float* gs_other,
                       float* gs_out, float* alpha_out, void* packed, void* sf_swizzled, void* workspace,
                       void* stream) {
  if (!x || !packed || !sf_swizzled || !workspace) return NVFP4_ERR_INVALID_VALUE;
  if (rows < 1 || k < 16 || k % 16) return NVFP4_ERR_INVALID_VALUE;
  if (in_dtype < NVFP4_DTYPE_F16 || in_dtype > NVFP4_DTYPE_F32) return NVFP4_ERR_INVALID_VALUE;
  if (alpha_out != nullptr && gs_other == nullptr) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned(x, 16) || !aligned(packed, 8) || !aligned(workspace, 4)) return NVFP4_ERR_MISALIGNED;
  if (!aligned(gs_other, 4) || !aligned(gs_out, 4) || !aligned(alpha_out, 4)) return NVFP4_ERR_MISALIGNED;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  DeviceCache* d = nullptr;
  rc = device_cache(dev, &d);
  if (rc != NVFP4_OK) return rc;
  if (d->cc_major != 10) return NVFP4_ERR_UNSUPPORTED;
  static_assert(g3::kActMaxParts * 4 <= NVFP4_ACT_WORKSPACE_BYTES, "act workspace");
  g3::QuantParams p;
  p.x = x;
  p.rows = rows;
  p.k = k;
  p.cols = k / 16;
  p.rows_pad = (rows + 127) / 128 * 128;
  p.cols_pad = (p.cols + 3) / 4 * 4;
  p.gs = 1.0f;
  p.gs_dev = nullptr;
  p.gs_mode = 2;
  p.div_mode = 0;  // CUDA torch: multiply by fl(1/6)
  p.packed = static_cast<uint8_t*>(packed);
  p.sf_swz = static_cast<uint8_t*>(sf_swizzled);
  p.sf_lin = nullptr;
  p.gs_out = gs_out;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // amax: two 16-element vectors per thread, at most kActMaxParts CTAs
  const int64_t nvec = rows * k / 16;
  int64_t parts = (nvec + 2 * g3::kActThreads - 1) / (2 * g3::kActThreads);
  const int64_t cap = static_cast<int64_t>(d->sm_count) * 4 < g3::kActMaxParts ? static_cast<int64_t>(d->sm_count) * 4
                                                                                : g3::kActMaxParts;
  if (parts > cap) parts = cap;
  if (parts < 1) parts = 1;
  uint32_t* ws = static_cast<uint32_t*>(workspace);
  switch (in_dtype) {
    case NVFP4_DTYPE_F16: g3::nvfp4_act_amax_kernel<0><<<static_cast<int>(parts), g3::kActThreads, 0, s>>>(x, rows * k, ws); break;
    case NVFP4_DTYPE_BF16: g3::nvfp4_act_amax_kernel<1><<<static_cast<int>(parts), g3::kActThreads, 0, s>>>(x, rows * k, ws); break;
    default: g3::nvfp4_act_amax_kernel<2><<<static_cast<int>(parts), g3::kActThreads, 0, s>>>(x, rows * k, ws); break;
  }
  G3_CUDA(cudaGetLastError());
  // For the few rows a weight-streaming GEMM follows (<= 128), at most one quantiser CTA per SM:
  // they become resident early (programmatic launch) and wait for the amax kernel, and each SM
  // must keep room for a GEMM CTA launched early the same way. Larger inputs get a full wave.
  const bool idx32 = quant_idx32(p);
  int qgrid = quant_grid(d, in_dtype, idx32 ? kQuantIdx32 : kQuantIdx64, p.rows_pad * p.cols_pad);
  if (rows <= 128 && qgrid > d->sm_count) qgrid = d->sm_count;
  cudaLaunchConfig_t lc = {};
  lc.gridDim = dim3(static_cast<unsigned>(qgrid), 1, 1);
  lc.blockDim = dim3(g3::kActThreads, 1, 1);
  lc.stream = s;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = &attr;
  lc.numAttrs = 1;
  const uint32_t* cparts = ws;
  const int nparts = static_cast<int>(parts);
  if (idx32) {
    switch (in_dtype) {
      case NVFP4_DTYPE_F16: G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_act_quantize_kernel<0, uint32_t>, p, cparts, nparts, gs_other, alpha_out)); break;
      case NVFP4_DTYPE_BF16: G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_act_quantize_kernel<1, uint32_t>, p, cparts, nparts, gs_other, alpha_out)); break;
      default: G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_act_quantize_kernel<2, uint32_t>, p, cparts, nparts, gs_other, alpha_out)); break;
    }
  } else {
    switch (in_dtype) {
      case NVFP4_DTYPE_F16: G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_act_quantize_kernel<0, int64_t>, p, cparts, nparts, gs_other, alpha_out)); break;
      case NVFP4_DTYPE_BF16: G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_act_quantize_kernel<1, int64_t>, p, cparts, nparts, gs_other, alpha_out)); break;
      default: G3_CUDA(cudaLaunchKernelEx(&lc, g3::nvfp4_act_quantize_kernel<2, int64_t>, p, cparts, nparts, gs_other, alpha_out)); break;
    }
  }
  return NVFP4_OK;
}

int nvfp4_dequantize(const void* packed, const void* sf_linear, int64_t rows, int64_t k, float global_scale,
                     int32_t div_mode, float* out, void* stream) {
  if (!packed || !sf_linear || !out || rows < 1 || k < 16 || k % 16) return NVFP4_ERR_INVALID_VALUE;
  if (div_mode != 0 && div_mode != 1) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned(packed, 8) || !aligned(out, 16)) return NVFP4_ERR_MISALIGNED;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  DeviceCache* d = nullptr;
  rc = device_cache(dev, &d);
  if (rc != NVFP4_OK) return rc;
  g3::DequantParams p;
  p.packed = static_cast<const uint8_t*>(packed);
  p.sf_lin = static_cast<const uint8_t*>(sf_linear);
  p.rows = rows;
  p.k = k;
  p.cols = k / 16;
  p.gs = global_scale;
  p.div_mode = div_mode;
  p.out = out;
  g3::nvfp4_dequantize_kernel<<<grid_for(rows * p.cols, d->sm_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(p);
  G3_CUDA(cudaGetLastError());
  return NVFP4_OK;
}

int nvfp4_swizzle_sf(const void* sf_linear, int64_t rows, int64_t cols, void* out, void* stream) {
  if (!sf_linear || !out || rows < 1 || cols < 1) return NVFP4_ERR_INVALID_VALUE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  DeviceCache* d = nullptr;
  rc = device_cache(dev, &d);
  if (rc != NVFP4_OK) return rc;
  const int64_t rp = (rows + 127) / 128 * 128, cp = (cols + 3) / 4 * 4;
  g3::nvfp4_swizzle_kernel<<<grid_for(rp * cp, d->sm_count), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(sf_linear), rows, cols, rp, cp, static_cast<uint8_t*>(out));
  G3_CUDA(cudaGetLastError());
  return NVFP4_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------
// Global-scale quantisation that allocates nothing.
//
// nvfp4_quantize with gs_mode 2 reads the tensor amax from a device float that the caller
// allocates and nvfp4_amax fills. Some callers cannot allocate it: a plugin or custom-call hook
// that a host framework hands only its input and output buffers, code running where cudaMalloc
// is not allowed (it can synchronise the device, and it is not legal while the stream is being
// captured), or a process whose memory is carved up in advance. nvfp4_quantize_global_noalloc
// keeps that intermediate in a fixed array of this library's own device memory instead.
namespace {

// Elements reduced by one block of the first pass, and how many per-block maxima the array holds;
// together they bound the input at 2^31 elements.
constexpr int64_t kNoAllocChunk = 65536;
constexpr int kNoAllocPartials = 32768;
static_assert(kNoAllocChunk * kNoAllocPartials == NVFP4_NOALLOC_MAX_ELEMENTS, "header limit out of sync");

// Words [0, kNoAllocPartials): per-block max |x| as FP32 bits; word kNoAllocPartials: the tensor
// amax read by the quantiser. 131,328 bytes, present on every device that loads this library
// until the process exits. Host code must not pass this name to a kernel (on the host it is only
// a stand-in); noalloc_scratch() gets the device address.
static __device__ __align__(256) uint32_t g_noalloc_scratch[kNoAllocPartials + 64];

uint32_t* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on `dev` (which must be current), looked up on the first
// call for that device and cached.
int noalloc_scratch(int dev, uint32_t** out) {
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    G3_CUDA(cudaGetSymbolAddress(&p, g_noalloc_scratch));
    if (p == nullptr) return NVFP4_ERR_CUDA;
    g_noalloc_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return NVFP4_OK;
}

// Pass 1: block b writes max |x| over elements [b * kNoAllocChunk, (b + 1) * kNoAllocChunk) to
// partials[b] as FP32 bits (NaN bits order above +Inf, so a NaN wins, as in nvfp4_amax_kernel).
// numel is a multiple of 16.
template <int kInDtype>
__global__ void __launch_bounds__(256) noalloc_partial_amax_kernel(const void* x, int64_t numel, uint32_t* partials) {
  const int64_t begin = static_cast<int64_t>(blockIdx.x) * kNoAllocChunk;
  const int64_t end = begin + kNoAllocChunk < numel ? begin + kNoAllocChunk : numel;
  uint32_t m = 0;
  for (int64_t e = begin + static_cast<int64_t>(threadIdx.x) * 16; e < end; e += 256 * 16) {
    float v[16];
    g3::load16<kInDtype>(x, e, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) m = max(m, __float_as_uint(v[i]) & 0x7FFFFFFFu);
  }
  __shared__ uint32_t warp_max[8];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
#pragma unroll
    for (int w = 1; w < 8; ++w) m = max(m, warp_max[w]);
    partials[blockIdx.x] = m;
  }
}

// Pass 2: scratch[kNoAllocPartials] = max of the `parts` partials just written by pass 1.
__global__ void __launch_bounds__(1024) noalloc_final_amax_kernel(uint32_t* scratch, int parts) {
  uint32_t m = 0;
  for (int i = threadIdx.x; i < parts; i += 1024) m = max(m, scratch[i]);
  __shared__ uint32_t warp_max[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = warp_max[threadIdx.x];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (threadIdx.x == 0) scratch[kNoAllocPartials] = m;
  }
}

}  // namespace

extern "C" int nvfp4_quantize_global_noalloc(const void* x, int32_t in_dtype, int64_t rows, int64_t k, void* packed,
                                             void* sf_swizzled, void* sf_linear, float* gs_out, void* stream) {
  if (!x || !packed || !sf_swizzled) return NVFP4_ERR_INVALID_VALUE;
  if (rows < 1 || k < 16 || k % 16) return NVFP4_ERR_INVALID_VALUE;
  if (in_dtype < NVFP4_DTYPE_F16 || in_dtype > NVFP4_DTYPE_F32) return NVFP4_ERR_INVALID_VALUE;
  if (!aligned(x, 16) || !aligned(packed, 8)) return NVFP4_ERR_MISALIGNED;
  if (rows > NVFP4_NOALLOC_MAX_ELEMENTS / k) return NVFP4_ERR_TOO_LARGE;
  int dev = 0;
  int rc = current_device(&dev);
  if (rc != NVFP4_OK) return rc;
  uint32_t* scratch = nullptr;
  rc = noalloc_scratch(dev, &scratch);
  if (rc != NVFP4_OK) return rc;
  // Every partial that pass 2 reads is written by pass 1 of the same call, and the amax word is
  // written by pass 2 before the quantiser reads it, so nothing needs clearing between calls.
  const int64_t numel = rows * k;
  const int parts = static_cast<int>((numel + kNoAllocChunk - 1) / kNoAllocChunk);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (in_dtype) {
    case NVFP4_DTYPE_F16: noalloc_partial_amax_kernel<0><<<parts, 256, 0, s>>>(x, numel, scratch); break;
    case NVFP4_DTYPE_BF16: noalloc_partial_amax_kernel<1><<<parts, 256, 0, s>>>(x, numel, scratch); break;
    default: noalloc_partial_amax_kernel<2><<<parts, 256, 0, s>>>(x, numel, scratch); break;
  }
  G3_CUDA(cudaGetLastError());
  noalloc_final_amax_kernel<<<1, 1024, 0, s>>>(scratch, parts);
  G3_CUDA(cudaGetLastError());
  return nvfp4_quantize(x, in_dtype, rows, k, 0.0f, reinterpret_cast<const float*>(scratch + kNoAllocPartials),
                        2, 0, packed, sf_swizzled, sf_linear, gs_out, stream);
}
