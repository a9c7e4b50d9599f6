/*
 * C ABI of libgemm3_b200.so: a B200 (sm_100a) NVFP4 block-scaled GEMM and its quantiser.
 *
 * Every entry point takes plain device pointers, element counts and a cudaStream_t passed as
 * void* (NULL = legacy default stream), returns an nvfp4_status code, launches asynchronously on
 * that stream and never allocates device memory. Buffers are owned by the caller.
 *
 * Data formats (the layout of the nvfp4_gemm_cute package, nvfp4_gemm_cute/quant.py:1-7):
 *   packed operand  uint8 [rows, K/2], row-major; element 2j in the low nibble, 2j+1 in the high
 *                   nibble; each nibble is an E2M1 code (bit 3 = sign, bits 0-2 index
 *                   {0, .5, 1, 1.5, 2, 3, 4, 6}).
 *   linear scales   uint8 [rows, K/16], UE4M3 bits, one per 16 consecutive K elements.
 *   swizzled scales uint8, ceil(rows/128)*128 * ceil(K/64)*4 bytes: rows padded to 128 and scale
 *                   columns to 4, each (128-row, 4-column) block stored as [32][4][4]
 *                   (row % 32, (row % 128) / 32, column % 4); blocks ordered row-block-major.
 */
#ifndef GEMM3_B200_NVFP4_GEMM_H_
#define GEMM3_B200_NVFP4_GEMM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes. Host-side validation failures are reported before anything is launched. */
typedef enum nvfp4_status {
  NVFP4_OK = 0,
  NVFP4_ERR_INVALID_VALUE = 1,   /* bad shape, null pointer or unsupported dtype */
  NVFP4_ERR_MISALIGNED = 2,      /* pointer alignment requirement violated */
  NVFP4_ERR_UNSUPPORTED = 3,     /* device is not sm_100 / feature not available */
  NVFP4_ERR_CUDA = 4,            /* a CUDA runtime call failed; see nvfp4_last_cuda_error() */
  NVFP4_ERR_TENSOR_MAP = 5,      /* cuTensorMapEncodeTiled rejected the operand */
  NVFP4_ERR_TOO_LARGE = 6,       /* input exceeds NVFP4_NOALLOC_MAX_ELEMENTS (no-allocation variant) */
  /* Device-side status words (written by kernels into the caller's int32 status buffer). */
  NVFP4_DEV_TIMEOUT_FULL = 101,
  NVFP4_DEV_TIMEOUT_EMPTY = 102,
  NVFP4_DEV_TIMEOUT_ACC_FULL = 103,
  NVFP4_DEV_TIMEOUT_ACC_EMPTY = 104,
  NVFP4_DEV_TIMEOUT_DRAIN = 105,
  NVFP4_DEV_ABORTED = 106
} nvfp4_status;

/* Element types of dense inputs/outputs. */
enum { NVFP4_DTYPE_F16 = 0, NVFP4_DTYPE_BF16 = 1, NVFP4_DTYPE_F32 = 2 };

/* L2 eviction priority hints for the operand loads. */
enum { NVFP4_L2_NORMAL = 0, NVFP4_L2_EVICT_FIRST = 1, NVFP4_L2_EVICT_LAST = 2 };

/*
 * Launch configuration of the GEMM kernel. Zero-initialise and set struct_size; zero fields take
 * their defaults. The library reads the first struct_size bytes, so a caller built against an
 * older, shorter struct gets defaults for the fields added since. Mirrors the attributes of nvfp4_gemm_cute.presets.Config
 * (nvfp4_gemm_cute/presets.py:14-35, api.py:20-39) that have a meaning on B200.
 */
typedef struct nvfp4_gemm_config {
  int32_t struct_size;           /* sizeof(nvfp4_gemm_config) */
  int32_t tile_m;                /* 256 (or 0): CTA pairs, 256x256 tiles; 128: one CTA per 128x256 tile */
  int32_t tile_n;                /* 256 (or 0); 128 with tile_m 128: weight-streaming kernel for M <= 128,
                                    128 rows of B (columns of C) per tile, all of A's rows in the MMA's N */
  int32_t raster_band;           /* 128-row tiles per raster band (0 or 1: bands of one tile) */
  int32_t raster_along_m;        /* 0: bands of M-tiles, sweep N ("N sweep"); 1: bands of N-tiles */
  int32_t l2_policy_a;           /* NVFP4_L2_* for A loads */
  int32_t l2_policy_b;
  int32_t l2_policy_sfa;
  int32_t l2_policy_sfb;
  int32_t store_evict_first;     /* output stores with L2::evict_first: 0 auto (K >= 8192), 1 on, 2 off */
  int32_t epi_store_pace_ns;     /* pause between output 32-column chunks (0 = none) */
  int32_t tma_b_first;           /* issue the B load before A in each stage */
  int32_t max_ctas;              /* cap on persistent CTAs (0 = one per SM) */
  int32_t pdl;                   /* programmatic dependent launch (nvfp4_gemm_cute/kernel.py:524):
                                    0 off; 1 the kernel's set-up overlaps the preceding kernel and
                                    every global read or write waits for it (griddepcontrol.wait);
                                    2 as 1, except that the weight-streaming kernel loads B and its
                                    scales before that wait (B must not be written by the preceding
                                    kernel; the other kernels treat 2 as 1). The CTA-pair and one-CTA
                                    kernels also let the next PDL launch start early. */
} nvfp4_gemm_config;

/*
 * C[M,N] = alpha * dequant(A)[M,K] . dequant(B)[N,K]^T, FP32 accumulation, FP16/BF16 output.
 * Replaces the TVM-FFI callable that nvfp4_gemm_cute/api.py:219 invokes
 *   compiled(a, b, out, sf_m, sf_n, sf_k, a_sf_ptr, b_sf_ptr, alpha)
 * (kernel wrapper at nvfp4_gemm_cute/kernel.py:1801-1870).
 *   a, b      packed operands, 16-byte aligned
 *   sfa, sfb  swizzled scales, 16-byte aligned
 *   c         contiguous [M,N] of out_dtype (NVFP4_DTYPE_F16 or _BF16), 32-byte aligned
 *   alpha     device pointer to one float (read on the device, like kernel.py:671)
 *   status    optional device int32 that receives the first device-side error (may be NULL)
 * Requires M >= 1, N % 64 == 0, K % 64 == 0 (api.py:173-174). cfg may be NULL (defaults).
 */
int nvfp4_gemm_run(const void* a, const void* b, const void* sfa, const void* sfb, void* c,
                   const float* alpha, int64_t m, int64_t n, int64_t k, int32_t out_dtype,
                   const nvfp4_gemm_config* cfg, int32_t* status, void* stream);

/* Destinations of nvfp4_gemm_run_gather: this GPU's buffer and up to 7 other GPUs' buffers. */
#define NVFP4_MAX_GATHER_DST 8
#define NVFP4_IPC_HANDLE_BYTES 64

/*
 * Column-parallel GEMM with the gather of C fused into the epilogue. Computes this rank's block
 * alpha * A . B^T (B holding the rank's N rows) and writes it as columns [col0, col0 + N) of
 * every row-major [M, ldc] buffer in c_dst[0..n_dst): c_dst[0] on this GPU (32-byte aligned),
 * c_dst[1..] other GPUs' buffers mapped into this process (nvfp4_ipc_open; 16-byte aligned),
 * reached with plain 16-byte stores over NVLink. It replaces the all-gather of the [M, N/g]
 * blocks and their relayout into row-major [M, N] that follow nvfp4_gemm_run on each rank.
 * Requires ldc >= col0 + N, ldc % 16 == 0, col0 % 16 == 0, 1 <= n_dst <= NVFP4_MAX_GATHER_DST;
 * other arguments as nvfp4_gemm_run. The kernel ends with a system-scope fence after its peer
 * stores; readers of a buffer must still be ordered after every rank's call (for example a
 * collective on each rank's stream after the GEMM). No counterpart in the reference, which is
 * single-GPU; it is the optional gather of the column-parallel GEMM.
 */
int nvfp4_gemm_run_gather(const void* a, const void* b, const void* sfa, const void* sfb, void* const* c_dst,
                          int32_t n_dst, int64_t ldc, int64_t col0, const float* alpha, int64_t m, int64_t n,
                          int64_t k, int32_t out_dtype, const nvfp4_gemm_config* cfg, int32_t* status,
                          void* stream);

/*
 * CUDA IPC for the gather's destinations (no counterpart in the reference). get_handle exports the
 * allocation that contains `ptr` (NVFP4_IPC_HANDLE_BYTES into `handle`) and ptr's offset in it;
 * another process opens it with nvfp4_ipc_open (peer access enabled on demand) and releases the
 * mapping with nvfp4_ipc_close(ptr, offset).
 */
int nvfp4_ipc_get_handle(const void* ptr, void* handle, int64_t* offset);
int nvfp4_ipc_open(const void* handle, int64_t offset, void** ptr);
int nvfp4_ipc_close(void* ptr, int64_t offset);

/*
 * Quantise x [rows, K] (contiguous, in_dtype F16/BF16/F32, 16-byte aligned) to NVFP4.
 * Replaces quantize_nvfp4 (nvfp4_gemm_cute/quant.py:41-59), bit-exact with it:
 *   xb = float(x) * gs;  amax over 16;  scale = e4m3_rn_nonsaturating(amax / 6);
 *   q = scale > 0 ? xb / scale : 0;  code = nearest E2M1 (ties to the even code) | sign(q < 0).
 * gs_mode selects the global scale gs:
 *   0: the host value global_scale;
 *   1: *gs_dev (device float);
 *   2: 2688 / *gs_dev where *gs_dev holds the tensor amax (from nvfp4_amax); gs = 1 if amax is 0
 *      or not finite. The gs used is written to gs_out when gs_out is not NULL.
 * div_mode selects how "amax / 6" rounds, matching where the reference ran:
 *   0: amax * fl(1/6) (PyTorch on CUDA divides by a host scalar through its reciprocal);
 *   1: correctly rounded amax / 6 (PyTorch on CPU).
 * Outputs: packed [rows, K/2]; sf_swizzled (padding written as zeros); sf_linear [rows, K/16]
 * (may be NULL). Requires K % 16 == 0 and packed 8-byte aligned. For F16/BF16 input with
 * K % 32 == 0, packed 16-byte aligned and both scale arrays 2-byte aligned, one thread
 * converts two neighbouring 16-element blocks (wider loads and stores; the same bytes).
 */
int nvfp4_quantize(const void* x, int32_t in_dtype, int64_t rows, int64_t k, float global_scale,
                   const float* gs_dev, int32_t gs_mode, int32_t div_mode, void* packed,
                   void* sf_swizzled, void* sf_linear, float* gs_out, void* stream);

/* Device workspace that nvfp4_quantize_act needs (per-CTA partial maxima; overwritten). */
#define NVFP4_ACT_WORKSPACE_BYTES 4096

/*
 * Quantise activations x [rows, K] with their tensor-wide global scale for an LLM projection
 * call: two launches on `stream` (an amax pass writing per-CTA partial maxima to `workspace`,
 * then the quantiser), chained by programmatic dependent launch. Equivalent, bit for bit, to
 * nvfp4_amax followed by nvfp4_quantize with gs_mode 2 and div_mode 0:
 *   gs = 2688 / amax(|x|) (1 if amax is 0, Inf or NaN), written to *gs_out when gs_out != NULL;
 *   packed codes [rows, K/2] and swizzled scales as nvfp4_quantize writes them.
 * It replaces the reference's quantize_nvfp4(x, global_scale=gs) (nvfp4_gemm_cute/quant.py:41-59)
 * with the global-scale recipe of nvfp4_gemm_cute/docs/usage.md:14, and also writes
 *   *alpha_out = 1 / (gs * *gs_other)  (FP32, correctly rounded)
 * when alpha_out != NULL: the GEMM alpha for weights quantised with global scale *gs_other (a
 * device float). workspace: NVFP4_ACT_WORKSPACE_BYTES of device memory, 4-byte aligned, not
 * shared with a concurrent call. Both kernels let the next launch in the stream start early: a
 * following nvfp4_gemm_run with cfg->pdl = 2 streams its weights while they run and waits for
 * them before reading A, A's scales or alpha.
 */
int nvfp4_quantize_act(const void* x, int32_t in_dtype, int64_t rows, int64_t k, const float* gs_other,
                       float* gs_out, float* alpha_out, void* packed, void* sf_swizzled, void* workspace,
                       void* stream);

/*
 * amax_out[0] = max |x| over numel elements (NaN propagates). No counterpart in the reference
 * package; it produces the per-tensor amax from which the FP32 global encode scale
 * 2688 / amax (= 1 / (amax / (6 * 448))) is derived for nvfp4_quantize gs_mode 2.
 */
int nvfp4_amax(const void* x, int32_t in_dtype, int64_t numel, float* amax_out, void* stream);

/*
 * nvfp4_amax followed by nvfp4_quantize in gs_mode 2 (div_mode 0), without the caller-allocated
 * amax float in between. No counterpart in the reference package.
 *
 * For callers that cannot allocate device memory: a plugin or custom-call hook that its host
 * framework hands only input and output buffers, code that may not call cudaMalloc because it
 * can synchronise the device or because a stream capture is open, or a process whose device
 * memory is all reserved up front. The amax intermediate lives instead in a fixed array of this
 * library's device memory (131,328 bytes, held on each device that loads the library until the
 * process exits). Outputs are bit-identical to nvfp4_amax + nvfp4_quantize(gs_mode 2, div_mode 0);
 * the gs used is written to gs_out when it is not NULL.
 *
 * - rows * k must not exceed NVFP4_NOALLOC_MAX_ELEMENTS (2^31); larger inputs return
 *   NVFP4_ERR_TOO_LARGE before anything is launched.
 * - The first call on a device looks up the array's device address (cudaGetSymbolAddress) with
 *   that device current; make that first call before any stream capture.
 * - Every call, on any stream, uses the same array: calls on one device whose kernels overlap on
 *   the GPU race and give wrong scales. Order them on one stream or with events. Nothing in the
 *   array needs to start at zero; each call writes what it reads.
 * - Calls no cudaMalloc, cudaFree or other allocating routine.
 */
#define NVFP4_NOALLOC_MAX_ELEMENTS 2147483648LL
int nvfp4_quantize_global_noalloc(const void* x, int32_t in_dtype, int64_t rows, int64_t k,
                                  void* packed, void* sf_swizzled, void* sf_linear, float* gs_out,
                                  void* stream);

/*
 * out[rows, K] (float32) = E2M1(code) * e4m3(scale) / global_scale.
 * Replaces dequantize_nvfp4 (nvfp4_gemm_cute/quant.py:62-70); div_mode as for nvfp4_quantize
 * (0: multiply by fl(1/gs) as PyTorch on CUDA does, 1: divide as PyTorch on CPU does).
 */
int nvfp4_dequantize(const void* packed, const void* sf_linear, int64_t rows, int64_t k,
                     float global_scale, int32_t div_mode, float* out, void* stream);

/* Linear [rows, cols] scales -> 128x4 swizzled layout, zero padded. Replaces swizzle_sf
 * (nvfp4_gemm_cute/quant.py:31-38). */
int nvfp4_swizzle_sf(const void* sf_linear, int64_t rows, int64_t cols, void* out, void* stream);

/* How many clusters of cluster_size CTAs of the default GEMM kernel (the CTA-pair kernel that
 * gemm() launches for tile 256x256, with its threads and shared memory) can be co-resident on the
 * current device; cluster_size 2 is the pair grid it launches. Replaces get_max_active_clusters
 * (nvfp4_gemm_cute/hw.py:8-22). */
int nvfp4_max_active_clusters(int32_t cluster_size, int32_t* out);

/* SM count, compute capability and L2 size of `device`. */
int nvfp4_device_info(int32_t device, int32_t* sm_count, int32_t* cc_major, int32_t* cc_minor,
                      int64_t* l2_bytes);

/* Set cudaLimitPersistingL2CacheSize of the current context to `bytes`, returning the previous
 * value in *old_bytes. Replaces the cudaDeviceSetLimit call of persisting_l2
 * (nvfp4_gemm_cute/api.py:223-242). A per-context limit: it ends with the process. */
int nvfp4_set_persisting_l2(int64_t bytes, int64_t* old_bytes);

/*
 * Failure-detection self-test; no counterpart in the reference. Launches one thread that waits,
 * through the bounded wait every GEMM kernel uses, on an mbarrier that nothing arrives at. After
 * the wait limit (2 s) it writes `code` (one of NVFP4_DEV_*) to the device int32 *status, if
 * *status is still 0, and the kernel exits; the context stays usable. Lets a test check that a
 * wait which cannot complete ends with a status instead of a hang.
 */
int nvfp4_selftest_wait_timeout(int32_t* status, int32_t code, void* stream);

/* Human-readable text for a status code; static storage. */
const char* nvfp4_strerror(int32_t code);

/* The cudaError_t of the most recent failing CUDA call on this thread (0 if none). */
int32_t nvfp4_last_cuda_error(void);

/* ABI version: bumped when a signature or struct layout changes. */
int32_t nvfp4_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* GEMM3_B200_NVFP4_GEMM_H_ */
