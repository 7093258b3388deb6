// Device-side building blocks shared by the NVFP4 kernels (sm_100a only):
// FP4/E4M3 conversions, the TE-compatible Philox4x32-10 counter stream,
// mbarrier / TMA / tcgen05 wrappers with bounded waits.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>

#if defined(__CUDA_ARCH__) && !defined(__CUDA_ARCH_FEAT_SM100_ALL)
#error "nvfp4_b200 device code targets sm_100a only (-gencode arch=compute_100a,code=sm_100a)"
#endif

namespace nvfp4 {

// ---------------------------------------------------------------------------
// Error word written by kernels whose bounded waits gave up.  One per device
// (file-scope __device__ in rht_gemm_sm100.cu); read by nvfp4_device_error().
// ---------------------------------------------------------------------------
enum DeviceError : uint32_t {
  kErrNone = 0,
  kErrTimeoutProducer = 1,
  kErrTimeoutMma = 2,
  kErrTimeoutEpilogue = 3,
  kErrTimeoutDrain = 4,
  kErrTimeoutExchange = 5,
  kErrTimeoutGridBarrier = 6,
};

// ---------------------------------------------------------------------------
// Scalar conversions
// ---------------------------------------------------------------------------

// cvt.rs.satfinite.e2m1x4.f32 with the operands listed low element first:
// nibble k of the result holds x_k, rounded up in magnitude iff
// (|x_k| - lo) / (hi - lo) + r_k / 2^16 >= 1, where r_0 = rbits[23:16]:[7:0],
// r_2 = rbits[31:24]:[15:8] and r_1, r_3 are the bit-reversals of r_0, r_2
// (the rule the B200 follows, pinned against Transformer Engine's functions).
__device__ __forceinline__ uint16_t sr_e2m1x4(float x0, float x1, float x2, float x3,
                                              uint32_t rbits) {
  uint16_t r;
  asm volatile("cvt.rs.satfinite.e2m1x4.f32 %0, {%1, %2, %3, %4}, %5;"
               : "=h"(r)
               : "f"(x3), "f"(x2), "f"(x1), "f"(x0), "r"(rbits));
  return r;
}

// cvt.rn.satfinite.e2m1x2.f32: x0 in the low nibble, x1 in the high nibble.
__device__ __forceinline__ uint32_t rn_e2m1x2(float x0, float x1) {
  uint32_t r;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\tcvt.u32.u8 %0, t;\n\t}"
      : "=r"(r)
      : "f"(x0), "f"(x1));
  return r;
}

// Round x to bf16 (RNE) and back: cvt.rn.bf16x2.f32 on a pair.
__device__ __forceinline__ void bf16_round_pair(float& a, float& b) {
  uint32_t p;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(b), "f"(a));
  a = __uint_as_float(p << 16);
  b = __uint_as_float(p & 0xFFFF0000u);
}

// E4M3 (cvt.rn.satfinite.e4m3x2.f32) of a single value, and its exact decode
// through f16 (cvt.rn.f16x2.e4m3x2).
__device__ __forceinline__ uint32_t e4m3_encode(float x) {
  uint16_t h;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %1;" : "=h"(h) : "f"(x));
  return h & 0xFFu;
}
__device__ __forceinline__ float e4m3_decode(uint32_t code) {
  uint32_t h2;
  uint16_t c = (uint16_t)(code | (code << 8));
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(c));
  float f;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tcvt.f32.f16 %0, lo;\n\t}"
      : "=f"(f)
      : "r"(h2));
  return f;
}

__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float fmin_nan(float a, float b) {
  float r;
  asm("min.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float rcp_approx_ftz(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// S_enc = min_nanprop(448 * 6 / amax, FLT_MAX), or 1 when amax == 0 or the
// quotient is 0 (TE's ComputeGlobalEncodeScaleFP4).
__device__ __forceinline__ float global_encode_scale(float amax) {
  float s = fmin_nan(__fdiv_rn(2688.0f, amax), 3.402823466e38f);
  return (amax == 0.0f || s == 0.0f) ? 1.0f : s;
}

// ---------------------------------------------------------------------------
// Philox4x32-10 with Transformer Engine's state conventions: key = seed,
// counter (x, y, z, w) starts at (offset_lo, offset_hi, subseq_lo, subseq_hi)
// and advances by one per generate4() with carry x -> y -> z -> w.
// ---------------------------------------------------------------------------
struct Philox {
  uint32_t x, y, z, w, k0, k1;

  // Counter after init(seed, subseq, offset) followed by `skip` generate4()
  // calls.  The offset step keeps TE's early exit on the y carry.
  __device__ __forceinline__ void init(uint64_t seed, uint64_t subseq, uint64_t offset,
                                       uint32_t skip) {
    k0 = (uint32_t)seed;
    k1 = (uint32_t)(seed >> 32);
    x = 0; y = 0;
    z = (uint32_t)subseq;
    w = (uint32_t)(subseq >> 32);
    uint32_t olo = (uint32_t)offset, ohi = (uint32_t)(offset >> 32);
    x += olo;
    if (x < olo) ohi++;
    y += ohi;
    if (!(ohi <= y)) { if (++z == 0) ++w; }
    add(skip);
  }
  __device__ __forceinline__ void add(uint32_t v) {
    uint32_t nx = x + v;
    if (nx < x) { if (++y == 0) { if (++z == 0) ++w; } }
    x = nx;
  }
  __device__ __forceinline__ uint4 generate4() {
    uint32_t c0 = x, c1 = y, c2 = z, c3 = w, a = k0, b = k1;
#pragma unroll
    for (int r = 0; r < 10; ++r) {
      uint64_t p0 = (uint64_t)0xD2511F53u * c0;
      uint64_t p1 = (uint64_t)0xCD9E8D57u * c2;
      uint32_t n0 = (uint32_t)(p1 >> 32) ^ c1 ^ a;
      uint32_t n2 = (uint32_t)(p0 >> 32) ^ c3 ^ b;
      c1 = (uint32_t)p1;
      c3 = (uint32_t)p0;
      c0 = n0;
      c2 = n2;
      a += 0x9E3779B9u;
      b += 0xBB67AE85u;
    }
    add(1);
    return make_uint4(c0, c1, c2, c3);
  }
};

// ---------------------------------------------------------------------------
// Shared memory, mbarrier, TMA, tcgen05
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete, giving up after
// `limit_ns` or when another role raised *abort.  Returns false on give-up;
// the caller then stops issuing work.  No wait in these kernels is unbounded.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  volatile uint32_t* abort_flag,
                                                  uint64_t limit_ns, uint32_t err_code,
                                                  uint32_t* err_word) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (((++spins) & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > limit_ns) {
        *abort_flag = 1u;
        if (err_word) atomicCAS(err_word, 0u, err_code);
        return false;
      }
    }
  }
}

// System-scope relaxed store / load of 64 bits: for a flag word that carries
// all of its payload itself (no other data is published through it), so no
// ordering fence is needed -- only single-copy atomicity and visibility.
__device__ __forceinline__ void st_relaxed_sys_u64(unsigned long long* p, unsigned long long v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_relaxed_sys_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// Atomic add with acquire-release semantics at GPU scope: the arrival of a
// grid barrier (the block's earlier writes are visible to whoever sees the
// count, and the block sees the writes of those that arrived before it).
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void st_release_gpu_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_gpu_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2-D TMA tile load into shared memory, completing on an mbarrier (no
// multicast; the tensor map always describes this GPU's own memory).
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const void* tmap, uint32_t bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(bar), "r"(x), "r"(y)
      : "memory");
}
// 2-D TMA tile store from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_2d(const void* tmap, uint32_t src, int32_t x,
                                             int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.tile.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(tmap), "r"(src), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// tcgen05 (5th-generation tensor core, accumulators in tensor memory)
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] = A[smem] * B[smem]^T (enable_input_d = 0: the accumulator is
// overwritten, never accumulated).
__device__ __forceinline__ void tc_mma_f16_overwrite(uint32_t d_tmem, uint64_t a_desc,
                                                     uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(0u)
      : "memory");
}
// Arrive once on an mbarrier when all previously issued tcgen05 ops of this
// thread have completed.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive fp32 columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld_32cols(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// Shared-memory matrix descriptor for tcgen05.mma (sm_100 format, version 1).
// lbo/sbo in bytes; layout: 0 = no swizzle, 2 = 128-byte swizzle.
__device__ __forceinline__ uint64_t umma_smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo,
                                                   uint32_t layout) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

}  // namespace nvfp4
