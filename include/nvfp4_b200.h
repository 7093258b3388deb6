/*
 * nvfp4_b200.h -- C ABI of the B200 (sm_100a) NVFP4 quantization library.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream,
 * allocates no memory, launches asynchronously on `stream` and returns an
 * nvfp4_status (0 = OK) instead of aborting.  `nvfp4_stream_t` is the same
 * type as cudaStream_t (NULL = legacy default stream).
 *
 * Layout conventions (identical to the reference):
 *   A    m x n bf16, column-major: element (i, j) at A[i + m * j]
 *   B    16 x 16 bf16, row-major:  element (k, c) at B[k * 16 + c]
 *   C    m x n FP4 E2M1, row-major, two codes per byte, even column in the
 *        low nibble: element (i, j) in byte i * n / 2 + j / 2
 *   SFC  m x n/16 E4M3 scale factors, row-major: SFC[i * (n / 16) + j / 16]
 *   global_amax   device pointer to one float
 *   rng_state     device pointer to {seed, offset} (size_t[2]) or NULL
 */
#ifndef NVFP4_B200_H_
#define NVFP4_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#ifndef NVFP4_API
#define NVFP4_API __attribute__((visibility("default")))
#endif

typedef struct CUstream_st* nvfp4_stream_t;

enum nvfp4_status {
  NVFP4_OK = 0,
  NVFP4_ERR_INVALID_SHAPE = 1,    /* m % 128, n % 64, cols % 16, k_tile_size < 64 ... */
  NVFP4_ERR_INVALID_ARGUMENT = 2, /* NULL pointer, bad flag combination */
  NVFP4_ERR_MISALIGNED = 3,       /* a pointer misses the alignment TMA / vector I/O needs */
  NVFP4_ERR_CUDA = 4,             /* a CUDA runtime call failed (see nvfp4_last_cuda_error) */
  NVFP4_ERR_UNSUPPORTED_DEVICE = 5, /* not a compute capability 10.0 device */
  NVFP4_ERR_DEVICE_TIMEOUT = 6,   /* a kernel's bounded wait gave up (nvfp4_device_error) */
  NVFP4_ERR_SCRATCH_CAPACITY = 7  /* more work units than nvfp4_quantize_rht_fused_noalloc's
                                     built-in scratch counts (2^31 - 1) */
};

/* Human-readable text for a status code. */
NVFP4_API const char* nvfp4_status_string(int status);
/* The cudaError_t behind the last NVFP4_ERR_CUDA on this host thread. */
NVFP4_API int nvfp4_last_cuda_error(void);

/* ---------------------------------------------------------------------- */
/* RHT GEMM fused with the NVFP4 cast                                      */
/* ---------------------------------------------------------------------- */

/* Replaces rht_gemm_ntt_w_sfc<bf16, bf16, e2m1, ue4m3, SR, FM>
 * (rht_gemm/te_ref/hadamard_transform_cast_fusion_core.inc:513-644; same
 * positional order as rht_gemm/rht_gemm_sm120.cuh:321-334), with the two
 * template flags as trailing ints.  For every 16-column group g:
 *   C[:, 16g:16g+16] = NVFP4(A[:, 16g:16g+16] * B)
 * with one E4M3 scale per (row, group) derived from *global_amax, stochastic
 * rounding from Philox4x32-10 keyed by rng_state in TE's coordinate mapping
 * (bit-exact with the reference kernel), or round-to-nearest.
 * Requires m % 128 == 0, n % 64 == 0, k_tile_size >= 64, A and C 16-byte
 * aligned.  m == 0 or n == 0 is a no-op.  sm_count == 0 means "all SMs";
 * it caps the persistent grid like the reference's argument. */
NVFP4_API int nvfp4_rht_gemm_ntt_w_sfc(int m, int n, const void* A, const void* B, void* C,
                                       void* SFC, const float* global_amax,
                                       const size_t* rng_state, uint32_t sm_count,
                                       nvfp4_stream_t stream, int k_tile_size,
                                       int stochastic_rounding, int use_fast_math);

/* Shard of a larger matrix: this call's A / C / SFC hold columns
 * [n_offset, n_offset + n) of an m x n_total problem; stochastic rounding
 * uses the coordinates of the full problem, so concatenating the shards'
 * outputs along the column dimension reproduces the unsharded call bit for
 * bit.  n_offset must be a multiple of 64 * (min(n_total, k_tile_size) / 64).
 * No reference counterpart: the reference has no multi-GPU path. */
NVFP4_API int nvfp4_rht_gemm_ntt_w_sfc_sharded(int m, int n, const void* A, const void* B,
                                               void* C, void* SFC, const float* global_amax,
                                               const size_t* rng_state, uint32_t sm_count,
                                               nvfp4_stream_t stream, int k_tile_size,
                                               int stochastic_rounding, int use_fast_math,
                                               int n_offset, int n_total);

/* Cross-GPU amax exchange over peer memory (NVLink), fused into the cast.
 * One process per GPU.  Set-up (allocates; not on the hot path):
 *   nvfp4_exchange_create(rank, world, &ex, handle)  -- 64-byte CUDA IPC handle out
 *   (all-gather the handles across ranks in rank order)
 *   nvfp4_exchange_connect(ex, handles)              -- world x 64 bytes
 *   (barrier across ranks before the first launch)
 * Then each rank calls nvfp4_rht_gemm_ntt_w_sfc_sharded_exchange with its
 * own shard's amax; the kernel publishes it to every peer, combines all ranks'
 * values (NaN-propagating max) and quantizes with the global amax, which it
 * also writes to global_amax_out (may be NULL, may alias local_amax).  Every
 * rank must make the same sequence of calls; a rank that does not join makes
 * the others' kernels give up after 1 s (nvfp4_device_error reports 5).
 * No reference counterpart: the reference has no multi-GPU path. */
typedef struct nvfp4_exchange nvfp4_exchange;
NVFP4_API int nvfp4_exchange_create(int rank, int world, nvfp4_exchange** ex,
                                    void* ipc_handle_out);
NVFP4_API int nvfp4_exchange_connect(nvfp4_exchange* ex, const void* all_handles);
NVFP4_API int nvfp4_exchange_destroy(nvfp4_exchange* ex);
NVFP4_API int nvfp4_rht_gemm_ntt_w_sfc_sharded_exchange(
    int m, int n, const void* A, const void* B, void* C, void* SFC, const float* local_amax,
    float* global_amax_out, const size_t* rng_state, uint32_t sm_count, nvfp4_stream_t stream,
    int k_tile_size, int stochastic_rounding, int use_fast_math, int n_offset, int n_total,
    nvfp4_exchange* ex);

/* Global amax and cast in ONE kernel (no separate pre-pass).  One block per
 * SM (cooperative launch) runs two independent pipelines; in a first pass
 * they stream A through their TMA rings and take the NaN-propagating max of
 * |A|, the blocks meet at a grid barrier, and the cast then takes the units
 * in descending order, so that the tiles the first pass read last are
 * re-read from L2.  Writes the amax to *amax_out (device float, may be NULL).
 * Results equal nvfp4_amax_bf16 followed by nvfp4_rht_gemm_ntt_w_sfc.
 * `workspace` is nvfp4_fused_workspace_bytes() (32) bytes of device memory,
 * zeroed once before first use, never used by two launches at the same time;
 * each completed launch leaves it ready for the next (zero it again after a
 * launch that reported NVFP4_ERR_DEVICE_TIMEOUT).
 * No reference counterpart: the reference takes the amax as an input and has
 * no amax kernel; this is the fused form its callers would otherwise need. */
NVFP4_API size_t nvfp4_fused_workspace_bytes(void);
NVFP4_API int nvfp4_quantize_rht_fused(int m, int n, const void* A, const void* B, void* C,
                                       void* SFC, float* amax_out, const size_t* rng_state,
                                       uint32_t sm_count, nvfp4_stream_t stream, int k_tile_size,
                                       int stochastic_rounding, int use_fast_math,
                                       void* workspace);
/* nvfp4_quantize_rht_fused for callers that cannot allocate device memory.
 * No counterpart in the reference.  Some hosts own every byte of device
 * memory through their own pool and do not let a library call cudaMalloc
 * (it can synchronize the device and bypasses the pool), so they cannot
 * provide nvfp4_quantize_rht_fused's workspace.  This entry point takes the
 * same inputs and outputs but keeps that workspace in a 32-byte array built
 * into the library: every GPU that loads the library holds it until the
 * process exits, and no call allocates anything.
 *   - Limit: the array's 32-bit counters hand out at most 2^31 - 1 work units
 *     (128 x 256 tiles of A) per call; a larger problem is refused with
 *     NVFP4_ERR_SCRATCH_CAPACITY before anything is enqueued.
 *   - A refused call (bad shape, pointer, alignment or capacity) enqueues
 *     nothing on `stream`.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *     The looked-up address is kept per device; it is not valid after a
 *     cudaDeviceReset of that device.
 *   - All calls share the one array: calls that may overlap on the GPU (other
 *     streams, other host threads) race and must be serialized by the caller.
 *     Each call clears the counters and amax words it needs at zero (a
 *     24-byte cudaMemsetAsync on `stream`); the array otherwise keeps the
 *     last call's contents. */
NVFP4_API int nvfp4_quantize_rht_fused_noalloc(int m, int n, const void* A, const void* B,
                                               void* C, void* SFC, float* amax_out,
                                               const size_t* rng_state, uint32_t sm_count,
                                               nvfp4_stream_t stream, int k_tile_size,
                                               int stochastic_rounding, int use_fast_math);

/* The same for one rank's column shard; the kernel also combines the ranks'
 * amax over peer memory (see nvfp4_exchange_create). */
NVFP4_API int nvfp4_quantize_rht_fused_sharded_exchange(
    int m, int n, const void* A, const void* B, void* C, void* SFC, float* amax_out,
    const size_t* rng_state, uint32_t sm_count, nvfp4_stream_t stream, int k_tile_size,
    int stochastic_rounding, int use_fast_math, int n_offset, int n_total, nvfp4_exchange* ex,
    void* workspace);

/* Fixed-flag entry points with the signature of the reference test's
 * wrappers run_ref / run_ref_fast / run_ref_sr
 * (rht_gemm/test_compare_ref.cu:70-88): k_tile_size = 2048. */
NVFP4_API int nvfp4_run_rht(int m, int n, const void* A, const void* B, void* C, void* SFC,
                            const float* global_amax, const size_t* rng_state, uint32_t sm_count,
                            nvfp4_stream_t stream);
NVFP4_API int nvfp4_run_rht_fast(int m, int n, const void* A, const void* B, void* C, void* SFC,
                                 const float* global_amax, const size_t* rng_state,
                                 uint32_t sm_count, nvfp4_stream_t stream);
NVFP4_API int nvfp4_run_rht_sr(int m, int n, const void* A, const void* B, void* C, void* SFC,
                               const float* global_amax, const size_t* rng_state,
                               uint32_t sm_count, nvfp4_stream_t stream);

/* Replaces rht_gemm_ttt_wrapper (core.inc:648-678): calls the ntt entry with
 * m and n swapped, so A is read as n x m column-major (an m x n row-major
 * tensor) and C / SFC are n x m / n x m/16.  Default k_tile_size there: 1024. */
NVFP4_API int nvfp4_rht_gemm_ttt(int m, int n, const void* A, const void* B, void* C, void* SFC,
                                 const float* global_amax, const size_t* rng_state,
                                 uint32_t sm_count, nvfp4_stream_t stream, int k_tile_size,
                                 int stochastic_rounding, int use_fast_math);

/* ---------------------------------------------------------------------- */
/* Batch forms of the four stochastic-rounding device functions            */
/* (include/nvfp4_sr.cuh); one call of the device function per group.     */
/* ---------------------------------------------------------------------- */

/* cvt_fp32_to_fp4_4x_with_stochastic_rounding (stochastic_rounding/
 * compare.cuh:51-62, sr.sm120.cuh:187-194): group g reads in[4g..4g+3] as
 * (in01.x, in01.y, in23.x, in23.y) and rbits[g]; out[g] holds 4 nibbles, so
 * `out` is the packed FP4 stream of `in`. */
NVFP4_API int nvfp4_cvt_fp32_to_fp4_4x_sr(const float* in, const uint32_t* rbits, uint16_t* out,
                                          size_t ngroups, nvfp4_stream_t stream);
/* mul_cvt_fp32_to_fp4_4x_with_stochastic_rounding (te_ref ptx.cuh:660-689,
 * sr.sm120.cuh:153-177) with one float2 scale for all groups. */
NVFP4_API int nvfp4_mul_cvt_fp32_to_fp4_4x_sr(const float* in, float scale_x, float scale_y,
                                              const uint32_t* rbits, uint16_t* out,
                                              size_t ngroups, nvfp4_stream_t stream);
/* mul_cvt_bf16_to_fp4_4x_with_stochastic_rounding (ptx.cuh:563-598,
 * sr.sm120.cuh:112-142): group g reads 4 bf16 at in_bf16 + 8g bytes. */
NVFP4_API int nvfp4_mul_cvt_bf16_to_fp4_4x_sr(const void* in_bf16, float scale_x, float scale_y,
                                              const uint32_t* rbits, uint16_t* out,
                                              size_t ngroups, nvfp4_stream_t stream);
/* mul_cvt_bf16_to_fp4_8x_stochastic_rounding<float | bf16> (ptx.cuh:839-918,
 * sr.sm120.cuh:205-240): group g reads 8 bf16 and rbits[2g], rbits[2g+1];
 * with scale_is_bf16 the scale is rounded to bf16 first. */
NVFP4_API int nvfp4_mul_cvt_bf16_to_fp4_8x_sr(const void* in_bf16, float scale, int scale_is_bf16,
                                              const uint32_t* rbits, uint32_t* out, size_t ngroups,
                                              nvfp4_stream_t stream);

/* Row-wise NVFP4 quantization of a rows x cols row-major bf16 tensor
 * (cols % 16 == 0): per 16-element block, SFC = E4M3(block_amax * S_enc / 6)
 * with TE's formula (core.inc:450-467) and two 8x SR conversions with the
 * block's reciprocal scale and rbits[4b .. 4b+3].  C: rows x cols/2 bytes,
 * SFC: rows x cols/16.  The reference's caller of the 8x function (TE's
 * NVFP4 quantize kernel) is not vendored; this is its B200 form. */
NVFP4_API int nvfp4_quantize_rowwise_bf16_sr(int rows, int cols, const void* X,
                                             const float* global_amax, const uint32_t* rbits,
                                             void* C, void* SFC, nvfp4_stream_t stream);

/* Global amax (max |x|, NaN-propagating) of n bf16 values into *out (device
 * float).  Enqueues a 4-byte memset of *out and one kernel.  The reference
 * takes global_amax as an input (core.inc:374); this is the pre-pass that
 * produces it. */
NVFP4_API int nvfp4_amax_bf16(const void* x, size_t n, float* out, nvfp4_stream_t stream);

/* The same amax for a stream of steps, without the memset: *out must already
 * hold +0 (a zeroed word, or the `clear` of the previous chained call), and the
 * call sets *clear to +0 for the next one, so two words alternate between
 * consecutive steps (step i: out = w[i % 2], clear = w[(i + 1) % 2]; both
 * zeroed once before the first step).  The kernel is launched as a
 * programmatic dependent of the previous kernel of the stream: it reads x
 * while that kernel drains, and only the clearing of *clear waits for it to
 * complete.  So x must not be written by the previous kernel of the stream.
 * No reference counterpart (see nvfp4_amax_bf16). */
NVFP4_API int nvfp4_amax_bf16_chained(const void* x, size_t n, float* out, float* clear,
                                      nvfp4_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Scaled FP8 conversions (include/nvfp4_fp8.cuh) over batches of groups    */
/* ---------------------------------------------------------------------- */

/* Input element types and FP8 formats of the FP8 conversions. */
enum { NVFP4_DTYPE_F32 = 0, NVFP4_DTYPE_BF16 = 1, NVFP4_DTYPE_F16 = 2 };
enum { NVFP4_FP8_E4M3 = 0, NVFP4_FP8_E5M2 = 1 };

/* mul_cvt_2x (te_ref ptx.cuh:923-1062): group g converts input elements
 * 2g, 2g+1 (in_dtype) times the floatx2 at scale + g * scale_stride (stride
 * in floats; 0 = one scale for every group) into FP8 bytes 2g, 2g+1 of out.
 * Round to nearest even, saturating to the largest finite value. */
NVFP4_API int nvfp4_mul_cvt_fp8_2x(const void* in, int in_dtype, const float* scale,
                                   size_t scale_stride, void* out, int fp8_format,
                                   size_t ngroups, nvfp4_stream_t stream);
/* mul_cvt_4x (ptx.cuh:1172-1693): group g converts elements 4g .. 4g+3 into
 * bytes 4g .. 4g+3.  scale_width 2: a floatx2 (elements 0, 2 take .x and 1, 3
 * take .y); scale_width 4: a floatx4, one component per element. */
NVFP4_API int nvfp4_mul_cvt_fp8_4x(const void* in, int in_dtype, const float* scale,
                                   int scale_width, size_t scale_stride, void* out,
                                   int fp8_format, size_t ngroups, nvfp4_stream_t stream);
/* mul_cvt_4x with a floatx2 scale as built with the reference's
 * _LOOSE_PRECISION macro: cvt.rs.satfinite.{e4m3,e5m2}x4.f32 with the constant
 * random word 0x80008000 instead of round-to-nearest. */
NVFP4_API int nvfp4_mul_cvt_fp8_4x_loose(const void* in, int in_dtype, const float* scale,
                                         size_t scale_stride, void* out, int fp8_format,
                                         size_t ngroups, nvfp4_stream_t stream);

/* ---------------------------------------------------------------------- */
/* Diagnostics                                                             */
/* ---------------------------------------------------------------------- */

/* Reads (and with clear != 0 resets) the current device's error word that a
 * kernel sets when one of its bounded waits gives up.  Synchronizes the
 * device.  *code == 0 means no kernel gave up. */
NVFP4_API int nvfp4_device_error(uint32_t* code, int clear);

#ifdef __cplusplus
}
#endif

#endif /* NVFP4_B200_H_ */
