// RHT GEMM fused with the NVFP4 cast, written for B200 (sm_100a).
//
// Computes, for an m x n column-major bf16 matrix A and a 16 x 16 bf16 matrix B,
// C[:, 16g:16g+16] = A[:, 16g:16g+16] * B for every 16-column group g, then
// quantizes each (row, group) 16-vector to NVFP4: one E4M3 scale from the
// vector's amax and the global amax, sixteen E2M1 codes by stochastic rounding
// (Philox4x32-10 in Transformer Engine's coordinate mapping) or by
// round-to-nearest.  Results are bit-identical to TE's SM100 kernel
// (rht_gemm/te_ref/hadamard_transform_cast_fusion_core.inc:92-506).
//
// Design (warp-specialised, two CTAs per SM, each with its own pipeline, so
// that the two epilogues do not advance in lockstep).  With every SM in use
// the grid has one CTA per work unit and each running CTA takes the units of
// CTAs that have not started yet through cluster launch control
// (clusterlaunchcontrol.try_cancel), which balances the SMs and the two CTAs
// of an SM; otherwise (fewer SMs requested, or the fused kernel's cooperative
// launch) a persistent grid walks the units round-robin.
//   work unit   128 rows x 256 columns of A (one output tile)
//   warp 0      TMA producer: 128 x 64 bf16 sub-tiles (two 64 x 64 boxes,
//               128-byte swizzle) into a 4-stage shared-memory ring
//   warp 1      tcgen05.mma issuer: per sub-tile four M128 N16 K16 bf16 MMAs
//               (one per 16-column group) into a 2-stage TMEM ring of
//               128-column fp32 accumulators; owns the CTA's 256 TMEM columns
//   warps 2-9   epilogue: tcgen05.ld of two 32-column slices of its 32 TMEM
//               lanes per stage, bf16 round trip, amax, E4M3 scale,
//               reciprocal, Philox, cvt.rs / cvt.rn; FP4 bytes staged in a
//               swizzled 128 x 128 B tile that one TMA store writes out; scale
//               bytes staged and copied out in 16-byte rows.
// Every wait is bounded (1 s); a kernel that gives up records an error word
// and unwinds (drains its TMA loads and MMAs, frees TMEM) instead of hanging.
#include <cstdint>
#include <atomic>
#include <cstring>
#include <mutex>
#include <unordered_map>

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "launch_common.h"
#include "nvfp4_b200.h"
#include "nvfp4_device.cuh"

namespace nvfp4 {

// Error word of this device (see nvfp4_device_error).
__device__ uint32_t g_device_error_word;

namespace rht {

constexpr int kBM = 128;          // rows per tile = TMEM lanes
constexpr int kSubN = 64;         // columns per TMA sub-tile
constexpr int kUnitN = 256;       // columns per work unit / output tile
constexpr int kAccN = 128;        // fp32 columns per TMEM accumulator stage
constexpr int kStages = 4;        // shared-memory ring depth
constexpr int kAccStages = 2;     // 2 x 128 = half the TMEM columns (two CTAs per SM)
constexpr uint32_t kTmemCols = kAccStages * 128;
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 32 * kEpiWarps;
constexpr int kThreads = 32 * (2 + kEpiWarps);
constexpr uint32_t kStageBytes = kBM * kSubN * 2;        // 16 KiB
constexpr uint32_t kHalfBytes = kStageBytes / 2;         // one 64 x 64 box
constexpr uint32_t kCTileBytes = kBM * kUnitN / 2;       // 16 KiB
constexpr uint32_t kSfcTileBytes = kBM * kUnitN / 16;    // 2 KiB
constexpr uint64_t kWaitLimitNs = 1000000000ull;         // 1 s per wait

constexpr uint32_t kOffA = 0;
constexpr uint32_t kOffC = kOffA + kStages * kStageBytes;
constexpr uint32_t kOffSfc = kOffC + 2 * kCTileBytes;
constexpr uint32_t kOffB = kOffSfc + 2 * kSfcTileBytes;
constexpr int kClcSlots = 4;      // cluster-launch-control response ring
constexpr uint32_t kOffClc = kOffB + 512;                 // 16 B per response
constexpr uint32_t kOffBar = kOffClc + 16 * kClcSlots;
constexpr uint32_t kNumBars = 2 * kStages + 2 * kAccStages + 1 + 2 * kClcSlots + 1;
constexpr uint32_t kOffTab = kOffBar + 8 * kNumBars;    // 256 reciprocal scales
constexpr uint32_t kOffKey = kOffTab + 256 * 4;         // Philox key schedule, 10 x {k0, k1}
constexpr uint32_t kOffMisc = kOffKey + 128;
constexpr uint32_t kSmemBytes = kOffMisc + 32 + 1024;   // + alignment slack

// tcgen05 instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B,
// both MN-major, N = 16, M = 128.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | (1u << 15) | (1u << 16) |
                            ((16u >> 3) << 17) | ((128u >> 4) << 24);

// Unsigned division by a runtime constant d (1 <= d < 2^31) for numerators
// below 2^31: q = (umulhi(n, mul) + n) >> shift (round-up method of
// Granlund and Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994).
struct FastDiv {
  uint32_t mul, shift;
  __host__ __device__ __forceinline__ uint32_t div(uint32_t n) const {
#if defined(__CUDA_ARCH__)
    return (__umulhi(n, mul) + n) >> shift;
#else
    return (uint32_t)((((uint64_t)n * mul) >> 32) + n) >> shift;
#endif
  }
};
inline FastDiv make_fast_div(uint32_t d) {
  uint32_t l = 0;
  while ((1ull << l) < d) ++l;
  FastDiv f;
  f.mul = (uint32_t)(((1ull << 32) * ((1ull << l) - d)) / d + 1);
  f.shift = l;
  return f;
}

struct Params {
  int m, n;
  int tiles_m;        // m / 128
  int units;          // tiles_m * ceil(n / 256)
  int n_offset;       // column offset of this shard in the full problem
  uint32_t ktm;       // TE's K_TILE_MAX = min(n_total, k_tile_size) / 64
  FastDiv div_ktm;    // x / ktm
  FastDiv div_tiles_m;  // x / tiles_m
  int sfc_vec;        // bytes per SFC store: 16, 4 or 1
  const uint16_t* B;
  uint8_t* sfc;
  const float* amax;     // global amax, or this rank's amax when world > 1
  const size_t* rng;
  // Cross-GPU amax exchange over peer memory (world > 1): peers[q] is rank
  // q's slot array (2 x world 64-bit slots, double-buffered by epoch parity).
  const unsigned long long* const* peers;
  int rank, world;
  uint32_t epoch;
  float* amax_out;       // receives the combined amax (block 0), may be null
  // Fused kernel: workspace of kFusedWsWords 32-bit words (layout: kWs*
  // below).  Zeroed once before first use; each launch leaves it ready for
  // the next.
  uint32_t* ws;
  // 1: the grid has one CTA per work unit and running CTAs take the units of
  // CTAs not yet started through cluster launch control (dynamic balance);
  // 0: a persistent grid walks the units round-robin.
  int dynamic;
  // 1: B arrives by one TMA load (B 16-byte aligned); 0: warp 1 copies it.
  int b_tma;
};

constexpr int kMaxUnits = 0x7FFFFFFF;   // work units per launch (32-bit counts)
// Fused-kernel workspace words.  The unit counters hand out work units
// (first pass: ascending; second pass: descending).  The second-pass counter
// and the amax word alternate between two copies by launch generation, so
// that the next launch's copy can be cleared while this one's is in use.
constexpr int kWsArrive = 0;   // grid-barrier arrival count
constexpr int kWsCnt1 = 1;     // first-pass unit counter
constexpr int kWsCnt2 = 2;     // second-pass unit counters (2 words, by generation parity)
constexpr int kWsAmax = 4;     // combined amax bits (2 words, by generation parity)
constexpr int kWsGen = 6;      // grid-barrier generation (launches so far)
constexpr int kWsClearBytes = 24;   // words 0..5: the ones a fresh start needs at zero
constexpr int kFusedWsWords = 8;

// The global amax of this launch.  With world > 1: block 0 publishes
// {epoch, bits of this rank's amax} into slot `rank` of every rank's slot
// array (system-scope relaxed 64-bit stores over NVLink: the word carries its
// whole payload, so no release fence is needed), then every block polls
// its own rank's slots until all `world` of them carry this epoch and takes
// the bitwise max (amax >= 0, so integer order is value order and NaN wins).
// Slots alternate by epoch parity: a rank can be at most one launch ahead of
// a peer that is still reading (its next publish needs this rank's next
// launch, which starts only after this one ends).  The poll gives up after
// kWaitLimitNs, records kErrTimeoutExchange and returns NaN.
__device__ __forceinline__ float launch_amax(const Params& p, float local,
                                             volatile uint32_t* abort_flag, uint64_t limit_ns) {
  if (p.world <= 1) return local;
  const uint32_t par = p.epoch & 1u;
  if (blockIdx.x == 0) {
    const uint32_t bits = __float_as_uint(local);
    const unsigned long long val = ((unsigned long long)p.epoch << 32) | bits;
    for (int q = 0; q < p.world; ++q)
      st_relaxed_sys_u64(const_cast<unsigned long long*>(p.peers[q]) + par * p.world + p.rank, val);
  }
  const unsigned long long* mine = p.peers[p.rank] + par * p.world;
  uint32_t mx = 0;
  const uint64_t t0 = globaltimer_ns();
  for (int q = 0; q < p.world; ++q) {
    unsigned long long v = ld_relaxed_sys_u64(mine + q);
    while ((uint32_t)(v >> 32) != p.epoch) {
      if (globaltimer_ns() - t0 > limit_ns) {
        *abort_flag = 1u;
        atomicCAS(&g_device_error_word, 0u, (uint32_t)kErrTimeoutExchange);
        return __uint_as_float(0x7FFFFFFFu);
      }
      v = ld_relaxed_sys_u64(mine + q);
    }
    mx = max(mx, (uint32_t)v);
  }
  const float am = __uint_as_float(mx);
  if (blockIdx.x == 0 && p.amax_out != nullptr) *p.amax_out = am;
  return am;
}

// Work units: unit u = tm + tiles_m * un covers rows [128 tm, 128 tm + 128)
// and columns [256 un, 256 un + 256).  In the persistent schedule each CTA
// owns u = blockIdx.x, blockIdx.x + gridDim.x, ...; under cluster launch
// control it jumps to the unit of the CTA it cancelled.
struct UnitIter {
  int u, tm, un, step_m, step_n;
  __device__ __forceinline__ void init(const Params& p) {
    step_n = (int)p.div_tiles_m.div(gridDim.x);
    step_m = (int)gridDim.x - step_n * p.tiles_m;
    u = blockIdx.x;
    set(p);
  }
  __device__ __forceinline__ void set(const Params& p) {
    un = (int)p.div_tiles_m.div((uint32_t)u);
    tm = u - un * p.tiles_m;
  }
  // Continue with unit u (dynamic schedule); u < 0 ends the walk.
  __device__ __forceinline__ void jump(const Params& p, int nu) {
    u = nu < 0 ? p.units : nu;
    if (u < p.units) set(p);
  }
  __device__ __forceinline__ bool valid(const Params& p) const { return u < p.units; }
  __device__ __forceinline__ void next(const Params& p) {
    u += gridDim.x;
    tm += step_m;
    un += step_n;
    if (tm >= p.tiles_m) { tm -= p.tiles_m; ++un; }
  }
};

struct Unit {
  int tm, m0, n0, nsub, nacc;
};
__device__ __forceinline__ Unit unit_from(const Params& p, int tm, int un) {
  Unit t;
  t.tm = tm;
  t.m0 = tm * kBM;
  t.n0 = un * kUnitN;
  const int rem = (p.n - t.n0) / kSubN;
  t.nsub = rem < 4 ? rem : 4;
  t.nacc = (t.nsub + 1) / 2;
  return t;
}
__device__ __forceinline__ Unit unit_at(const Params& p, const UnitIter& it) {
  return unit_from(p, it.tm, it.un);
}
// Unit number u (u < p.units).
__device__ __forceinline__ Unit unit_of(const Params& p, int u) {
  const int un = (int)p.div_tiles_m.div((uint32_t)u);
  return unit_from(p, u - un * p.tiles_m, un);
}

__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// (a, b) * (s, s) with one mul.rn.f32x2: the same rounding as two mul.rn.f32.
__device__ __forceinline__ void mul2(float& a, float& b, float s) {
  uint64_t x, y;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a), "f"(b));
  asm("mov.b64 %0, {%1, %1};" : "=l"(y) : "f"(s));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(x) : "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(x));
}

// Shared-memory access by 32-bit shared-window address.
__device__ __forceinline__ void sts128(uint32_t addr, uint4 v) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ float lds_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}

// Two E2M1 x4 conversions by stochastic rounding packed into one word (the
// first four values in the low half).
__device__ __forceinline__ uint32_t sr_e2m1x8(float x0, float x1, float x2, float x3, float x4,
                                              float x5, float x6, float x7, uint32_t r0,
                                              uint32_t r1) {
  uint32_t w;
  asm("{\n\t.reg .b16 lo, hi;\n\t"
      "cvt.rs.satfinite.e2m1x4.f32 lo, {%4, %3, %2, %1}, %9;\n\t"
      "cvt.rs.satfinite.e2m1x4.f32 hi, {%8, %7, %6, %5}, %10;\n\t"
      "mov.b32 %0, {lo, hi};\n\t}"
      : "=r"(w)
      : "f"(x0), "f"(x1), "f"(x2), "f"(x3), "f"(x4), "f"(x5), "f"(x6), "f"(x7), "r"(r0), "r"(r1));
  return w;
}

// quant16 (TE's epilogue math, core.inc:439-492) on two adjacent 16-vectors
// of one row: writes their 32 FP4 codes to `out` (16 bytes) and returns both
// SFC codes as one 16-bit value, the first vector's in the low byte, from one
// cvt.rn.satfinite.e4m3x2.  `tab` is the shared-window address of the
// 256-entry reciprocal-scale table.
template <bool SR, bool FM>
__device__ __forceinline__ uint32_t quant32(float* x, float enc_mult, uint32_t tab, uint4 ra,
                                            uint4 rb, uint4& out) {
  if constexpr (!FM) {
#pragma unroll
    for (int k = 0; k < 32; k += 2) bf16_round_pair(x[k], x[k + 1]);
  }
  float a0 = max3_nan(fabsf(x[0]), fabsf(x[1]), fabsf(x[2]));
  float a1 = max3_nan(fabsf(x[16]), fabsf(x[17]), fabsf(x[18]));
#pragma unroll
  for (int k = 3; k < 15; k += 2) {
    a0 = max3_nan(a0, fabsf(x[k]), fabsf(x[k + 1]));
    a1 = max3_nan(a1, fabsf(x[16 + k]), fabsf(x[17 + k]));
  }
  a0 = fmax_nan(a0, fabsf(x[15]));
  a1 = fmax_nan(a1, fabsf(x[31]));
  uint32_t h;
  asm("{\n\t.reg .b16 t;\n\tcvt.rn.satfinite.e4m3x2.f32 t, %1, %2;\n\tcvt.u32.u16 %0, t;\n\t}"
      : "=r"(h)
      : "f"(a1 * enc_mult), "f"(a0 * enc_mult));
  const float s0 = lds_f32(tab + ((h & 0xFFu) << 2)), s1 = lds_f32(tab + ((h >> 8) << 2));
#pragma unroll
  for (int k = 0; k < 16; k += 2) mul2(x[k], x[k + 1], s0);
#pragma unroll
  for (int k = 16; k < 32; k += 2) mul2(x[k], x[k + 1], s1);
  if constexpr (SR) {
    out.x = sr_e2m1x8(x[0], x[1], x[2], x[3], x[4], x[5], x[6], x[7], ra.x, ra.y);
    out.y = sr_e2m1x8(x[8], x[9], x[10], x[11], x[12], x[13], x[14], x[15], ra.z, ra.w);
    out.z = sr_e2m1x8(x[16], x[17], x[18], x[19], x[20], x[21], x[22], x[23], rb.x, rb.y);
    out.w = sr_e2m1x8(x[24], x[25], x[26], x[27], x[28], x[29], x[30], x[31], rb.z, rb.w);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
      w[i] = rn_e2m1x2(x[8 * i], x[8 * i + 1]) | (rn_e2m1x2(x[8 * i + 2], x[8 * i + 3]) << 8) |
             (rn_e2m1x2(x[8 * i + 4], x[8 * i + 5]) << 16) |
             (rn_e2m1x2(x[8 * i + 6], x[8 * i + 7]) << 24);
    out = make_uint4(w[0], w[1], w[2], w[3]);
  }
  return h;
}

// Philox4x32-10 of the four counters (x0 + i, y, z, 0), i = 0..3, which
// differ only in their first word and do not carry out of it (x0 + 3 does
// not wrap).  Their first two rounds share work: round 0 multiplies the
// common z, round 1 the common first word it produced.  The key schedule
// {k0[r], k1[r]} is read from shared memory (`keys`, 16 bytes per two rounds).
__device__ __forceinline__ void philox4_shared(uint32_t x0, uint32_t y, uint32_t z, uint32_t keys,
                                               uint4 (&out)[4]) {
  constexpr uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u;
  uint32_t c0[4], c1[4], c2[4], c3[4];
  uint4 kk = lds128(keys);   // rounds 0 and 1
  const uint64_t q1 = (uint64_t)M1 * z;
  const uint32_t s0 = (uint32_t)(q1 >> 32) ^ y ^ kk.x;
  const uint32_t s1 = (uint32_t)q1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t q0 = (uint64_t)M0 * (x0 + (uint32_t)i);
    c2[i] = (uint32_t)(q0 >> 32) ^ kk.y;   // ^ w, w = 0
    c3[i] = (uint32_t)q0;
  }
  const uint64_t q0s = (uint64_t)M0 * s0;
  const uint32_t h0 = (uint32_t)(q0s >> 32), l0 = (uint32_t)q0s;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint64_t qq = (uint64_t)M1 * c2[i];
    c0[i] = (uint32_t)(qq >> 32) ^ s1 ^ kk.z;
    c1[i] = (uint32_t)qq;
    c2[i] = h0 ^ c3[i] ^ kk.w;
    c3[i] = l0;
  }
#pragma unroll
  for (int rp = 1; rp < 5; ++rp) {
    kk = lds128(keys + 16 * rp);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t ka = h ? kk.z : kk.x, kb = h ? kk.w : kk.y;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint64_t pa = (uint64_t)M0 * c0[i], pb = (uint64_t)M1 * c2[i];
        const uint32_t n0 = (uint32_t)(pb >> 32) ^ c1[i] ^ ka;
        const uint32_t n2 = (uint32_t)(pa >> 32) ^ c3[i] ^ kb;
        c1[i] = (uint32_t)pb;
        c3[i] = (uint32_t)pa;
        c0[i] = n0;
        c2[i] = n2;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) out[i] = make_uint4(c0[i], c1[i], c2[i], c3[i]);
}

// Philox4x32-10 for two consecutive counters (ctr and ctr + 1 in x with
// carry), with the key schedule read from shared memory as in philox4_shared.
__device__ __forceinline__ void philox_pair(uint32_t x, uint32_t y, uint32_t z, uint32_t w,
                                            uint32_t keys, uint4& ra, uint4& rb) {
  uint32_t a0 = x, a1 = y, a2 = z, a3 = w;
  uint32_t b0 = x + 1u, b1 = y, b2 = z, b3 = w;
  if (b0 == 0u) { if (++b1 == 0u) { if (++b2 == 0u) ++b3; } }
#pragma unroll
  for (int rp = 0; rp < 5; ++rp) {
    const uint4 kk = lds128(keys + 16 * rp);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t ka = h ? kk.z : kk.x, kb = h ? kk.w : kk.y;
      const uint64_t pa0 = (uint64_t)0xD2511F53u * a0, pa1 = (uint64_t)0xCD9E8D57u * a2;
      const uint64_t pb0 = (uint64_t)0xD2511F53u * b0, pb1 = (uint64_t)0xCD9E8D57u * b2;
      const uint32_t na0 = (uint32_t)(pa1 >> 32) ^ a1 ^ ka;
      const uint32_t na2 = (uint32_t)(pa0 >> 32) ^ a3 ^ kb;
      const uint32_t nb0 = (uint32_t)(pb1 >> 32) ^ b1 ^ ka;
      const uint32_t nb2 = (uint32_t)(pb0 >> 32) ^ b3 ^ kb;
      a1 = (uint32_t)pa1; a3 = (uint32_t)pa0; a0 = na0; a2 = na2;
      b1 = (uint32_t)pb1; b3 = (uint32_t)pb0; b0 = nb0; b2 = nb2;
    }
  }
  ra = make_uint4(a0, a1, a2, a3);
  rb = make_uint4(b0, b1, b2, b3);
}

// 4-D TMA tile load (the B matrix in its canonical no-swizzle layout).
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const void* tmap, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%3, %3, %3, %3}], [%2];" ::"r"(dst),
      "l"(tmap), "r"(bar), "r"(0)
      : "memory");
}

// Cluster launch control (one-CTA clusters): ask to cancel a CTA of this grid
// that has not started yet; the 16-byte response lands in shared memory and
// completes `bar` (transaction count 16).
__device__ __forceinline__ void clc_try_cancel(uint32_t resp, uint32_t bar) {
  asm volatile(
      "clusterlaunchcontrol.try_cancel.async.shared::cta.mbarrier::complete_tx::bytes.b128 "
      "[%0], [%1];" ::"r"(resp), "r"(bar)
      : "memory");
}
// The first CTA index a response names, or -1 if no CTA was cancelled.
__device__ __forceinline__ int clc_decode(uint32_t resp) {
  uint32_t x = 0, ok = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t.reg .b128 r;\n\t"
      "ld.shared.b128 r, [%2];\n\t"
      "clusterlaunchcontrol.query_cancel.is_canceled.pred.b128 p, r;\n\t"
      "selp.u32 %1, 1, 0, p;\n\t"
      "@p clusterlaunchcontrol.query_cancel.get_first_ctaid.v4.b32.b128 {%0, _, _, _}, r;\n\t}"
      : "+r"(x), "=r"(ok)
      : "r"(resp)
      : "memory");
  return ok ? (int)x : -1;
}

// Warp-uniform bounded wait: every lane polls the barrier (no divergent
// branch around the wait) and the warp agrees on the verdict with a vote.
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity,
                                          volatile uint32_t* abort_flag, uint32_t err) {
  const bool ok =
      mbar_wait_bounded(bar, parity, abort_flag, kWaitLimitNs, err, &g_device_error_word);
  return __all_sync(0xFFFFFFFFu, ok);
}

// ---------------------------------------------------------------------------
// Epilogue building blocks shared by the cast kernels
// ---------------------------------------------------------------------------

// Per-thread constants of an epilogue thread, set up once per CTA.
struct EpiThread {
  int r, g;               // row within the 128-row tile; this warp group's k-block of a stage
  uint32_t c_row, s_row;  // row r of the FP4 / SFC staging tiles, buffer 0 (shared window)
  uint32_t c_off[2][2];   // byte offset of chunk 4a + 2g + j within row r (128-byte swizzle)
  uint32_t t_row;         // TMEM lane r, column 64 g of accumulator stage 0
  uint32_t tab, keys;     // reciprocal-scale table, Philox key schedule (shared window)
  float enc_mult;         // S_enc / 6
  uint32_t olo, ohi;      // Philox counter offset
  bool chunk_aligned;     // K_TILE_MAX % 4 == 0: a unit's four k-blocks share one RNG chunk
};

// q: the TMEM lane quarter of this warp; c_tile / s_tile: shared-window
// addresses of staging buffer 0; tmem: the CTA's (or pipeline's) first
// accumulator column.
template <bool SR>
__device__ __forceinline__ EpiThread epi_setup(const Params& p, int q, int g, int lane,
                                               uint32_t c_tile, uint32_t s_tile, uint32_t tmem,
                                               uint32_t tab, uint32_t keys, float gamax) {
  EpiThread e;
  e.r = q * 32 + lane;
  e.g = g;
  // Row r of the 128 x 128 B FP4 staging tile holds the unit's columns in
  // 16-byte chunks, chunk c at position c ^ (r % 8) (128-byte swizzle).
  e.c_row = c_tile + (uint32_t)e.r * 128u;
  e.s_row = s_tile + (uint32_t)e.r * 16u + (uint32_t)g * 4u;
#pragma unroll
  for (int a = 0; a < 2; ++a)
#pragma unroll
    for (int j = 0; j < 2; ++j)
      e.c_off[a][j] = (((uint32_t)(a * 4 + 2 * g + j)) ^ (uint32_t)(e.r & 7)) * 16u;
  e.t_row = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)g * 64u;
  e.tab = tab;
  e.keys = keys;
  e.enc_mult = global_encode_scale(gamax) * (1.0f / 6.0f);
  e.olo = 0;
  e.ohi = 0;
  if constexpr (SR) {
    uint64_t offset = 0;
    if (p.rng != nullptr) offset = p.rng[1];
    e.olo = (uint32_t)offset;
    e.ohi = (uint32_t)(offset >> 32);
  }
  e.chunk_aligned = (p.ktm & 3u) == 0u;
  return e;
}

// The epilogue's share of one work unit: for each accumulator stage a, this
// warp group's k-block 2a + g: TE's Philox words, then the two 32-column
// slices of TMEM, quantized into the staging buffers `buf`.  Returns false
// when a wait gave up.
template <bool SR, bool FM>
__device__ __forceinline__ bool epi_cast_unit(const Params& p, const Unit& t, const EpiThread& e,
                                              uint32_t buf, uint32_t accf0, uint32_t acce0,
                                              uint32_t& acc, uint32_t& accph,
                                              volatile uint32_t* abort_flag) {
  const uint32_t cb = e.c_row + buf * kCTileBytes;
  const uint32_t sb = e.s_row + buf * kSfcTileBytes;
  // TE's RNG coordinates of this unit's first 64-column k-block
  // (core.inc:161-166, 470-475): kb / K_TILE_MAX and kb % K_TILE_MAX.
  const uint32_t kb0 = (uint32_t)((p.n_offset + t.n0) / kSubN);
  const uint32_t chunk0 = p.div_ktm.div(kb0);
  const uint32_t kt0 = kb0 - chunk0 * p.ktm;
  // TE's generate4() numbers 0..3 of sequence
  // seq = row + k_tile * 256 + linear_tile * K_TILE_MAX * 256 with
  // linear_tile = tile_m + tiles_m * chunk, counter (offset, seq, 0), for
  // k-block 2a + g of stage a.  When the unit's four k-blocks lie in one RNG
  // chunk, seq grows by 256 per block.
  const uint32_t seq0 = (uint32_t)e.r +
                        (kt0 + ((uint32_t)t.tm + (uint32_t)p.tiles_m * chunk0) * p.ktm) * 256u +
                        (uint32_t)e.g * 256u;
#pragma unroll
  for (int a = 0; a < 2; ++a) {
    if (a >= t.nacc) break;
    const int blk = 2 * a + e.g;
    // k-block beyond a ragged unit's end: computed on stale TMEM columns
    // (allocated, never written for this unit) and not stored
    const bool valid = blk < t.nsub;
    uint4 rw[4];
    if constexpr (SR) {
      // generated before waiting for the accumulator: overlaps the wait
      uint32_t seq = seq0 + (uint32_t)a * 512u;
      if (!e.chunk_aligned) {
        uint32_t kt = kt0 + (uint32_t)blk, chunk = chunk0;
        while (kt >= p.ktm) { kt -= p.ktm; ++chunk; }
        seq = (uint32_t)e.r + (kt + ((uint32_t)t.tm + (uint32_t)p.tiles_m * chunk) * p.ktm) * 256u;
      }
      if (e.olo <= 0xFFFFFFFCu) {
        philox4_shared(e.olo, e.ohi, seq, e.keys, rw);
      } else {
        // the counter's first word wraps within the four: carry each counter
        // separately
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t cx = e.olo + 2u * (uint32_t)j, cy = e.ohi, cz = seq, cw = 0;
          if (cx < e.olo) { if (++cy == 0u) { if (++cz == 0u) ++cw; } }
          philox_pair(cx, cy, cz, cw, e.keys, rw[2 * j], rw[2 * j + 1]);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 4; ++i) rw[i] = make_uint4(0, 0, 0, 0);
    }
    if (!warp_wait(accf0 + 8 * acc, accph, abort_flag, kErrTimeoutEpilogue)) return false;
    tc_fence_after();
    const uint32_t ta = e.t_row + acc * kAccN;
    uint32_t h0 = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      float v[32];
      tmem_ld_32cols(ta + j * 32, v);
      tc_wait_ld();
      if (j == 1) {
        // both slices are in registers: release the accumulator stage
        tc_fence_before();
        __syncwarp();
        mbar_arrive(acce0 + 8 * acc);
      }
      uint4 wq;
      const uint32_t h = quant32<SR, FM>(v, e.enc_mult, e.tab, rw[2 * j], rw[2 * j + 1], wq);
      if (valid) sts128(cb + e.c_off[a][j], wq);
      if (j == 0) h0 = h;
      else if (valid) sts32(sb + (uint32_t)a * 8u, h0 | (h << 16));
    }
    if (++acc == kAccStages) { acc = 0; accph ^= 1u; }
  }
  return true;
}

// A finished unit leaves the staging buffers: the leader thread issues the
// TMA store of the FP4 tile, warps 0-3 of the epilogue copy one 16-byte SFC
// row each.
__device__ __forceinline__ void epi_store_unit(const Params& p, const Unit& t,
                                               const CUtensorMap* tmC, uint32_t c_tile,
                                               const uint8_t* s_tile, int ew, int lane,
                                               bool leader) {
  if (leader) {
    tma_store_2d(tmC, c_tile, t.n0 / 2, t.m0);
    bulk_commit();
  }
  if (ew < 4) {
    const int row = ew * 32 + lane;
    uint8_t* dst = p.sfc + (size_t)(t.m0 + row) * (size_t)(p.n / 16) + t.n0 / 16;
    const uint8_t* src = s_tile + row * 16;
    const int nbytes = t.nsub * 4;
    if (p.sfc_vec == 16 && nbytes == 16) {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    } else if (p.sfc_vec >= 4) {
      for (int b = 0; b < nbytes; b += 4)
        *reinterpret_cast<uint32_t*>(dst + b) = *reinterpret_cast<const uint32_t*>(src + b);
    } else {
      for (int b = 0; b < nbytes; ++b) dst[b] = src[b];
    }
  }
}

template <bool SR, bool FM>
__global__ void __launch_bounds__(kThreads, 2)
    rht_nvfp4_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmC,
                     const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  // Launched as a programmatic dependent of the previous kernel in the
  // stream: the block is resident before that kernel has finished, and
  // waits here until it has completed and its writes are visible.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const uint32_t bar0 = sbase + kOffBar;
  auto full_bar = [&](uint32_t s) { return bar0 + 8 * s; };
  auto empty_bar = [&](uint32_t s) { return bar0 + 8 * (kStages + s); };
  auto accf_bar = [&](uint32_t a) { return bar0 + 8 * (2 * kStages + a); };
  auto acce_bar = [&](uint32_t a) { return bar0 + 8 * (2 * kStages + kAccStages + a); };
  const uint32_t drain_bar = bar0 + 8 * (2 * kStages + 2 * kAccStages);
  auto clcf_bar = [&](uint32_t s) { return bar0 + 8 * (2 * kStages + 2 * kAccStages + 1 + s); };
  auto clce_bar = [&](uint32_t s) {
    return bar0 + 8 * (2 * kStages + 2 * kAccStages + 1 + kClcSlots + s);
  };
  auto clc_resp = [&](uint32_t s) { return sbase + kOffClc + 16 * s; };
  // Unit number j >= 1 of this CTA under the dynamic schedule: the response of
  // request j (slot (j - 1) % kClcSlots).  Every role reads every response
  // once; -1 ends the walk (no CTA left to cancel, or a wait gave up).
  auto clc_slot = [](uint32_t j) { return (j - 1) % (uint32_t)kClcSlots; };
  auto clc_parity = [](uint32_t j) { return ((j - 1) / (uint32_t)kClcSlots) & 1u; };
  const uint32_t bfull_bar = bar0 + 8 * (kNumBars - 1);
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + kOffMisc);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + kOffMisc + 4);
  volatile int* next_unit = reinterpret_cast<volatile int*>(smem + kOffMisc + 16);

  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (uint32_t a = 0; a < kAccStages; ++a) {
      mbar_init(accf_bar(a), 1);
      mbar_init(acce_bar(a), kEpiThreads);   // every epilogue thread arrives
    }
    mbar_init(drain_bar, 1);
    mbar_init(bfull_bar, 1);
    for (uint32_t sl = 0; sl < (uint32_t)kClcSlots; ++sl) {
      mbar_init(clcf_bar(sl), 1);
      mbar_init(clce_bar(sl), 3);   // producer, MMA, epilogue warp 0
    }
    *abort_flag = 0u;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmC);
    if (p.b_tma) prefetch_tmap(&tmB);
  }
  float* acc_tab = reinterpret_cast<float*>(smem + kOffTab);
  float* s_amax = reinterpret_cast<float*>(smem + kOffMisc + 8);
  if (warp == 1) {
    if (!p.b_tma) {
      // B into shared memory in the canonical no-swizzle MN-major layout:
      // B(n = c, k) at (c % 8) * 2 + (k % 8) * 16 + (c / 8) * 128 + (k / 8) * 256.
      uint16_t* sb = reinterpret_cast<uint16_t*>(smem + kOffB);
      for (int idx = lane; idx < 256; idx += 32) {
        const int k = idx >> 4, c = idx & 15;
        const uint32_t off = (c & 7) * 2 + (k & 7) * 16 + (c >> 3) * 128 + (k >> 3) * 256;
        sb[off >> 1] = p.B[idx];
      }
      fence_proxy_async_smem();
    }
    tmem_alloc(smem_addr(tmem_holder), kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0;
      bool ok = true;
      if (p.b_tma) {
        // B in the canonical no-swizzle MN-major layout, straight from the
        // 4-D view (c % 8, k % 8, c / 8, k / 8) of the row-major 16 x 16 matrix.
        mbar_arrive_expect_tx(bfull_bar, 512);
        tma_load_4d(sbase + kOffB, &tmB, bfull_bar);
      }
      UnitIter it;
      uint32_t k = 0;               // index of the current unit
      bool pending = false;         // a cancel request whose response is unread
      for (it.init(p); it.valid(p) && ok;) {
        if (p.dynamic) {
          // request the unit after this one while this one streams in
          const uint32_t j = k + 1, sl = clc_slot(j);
          if (!mbar_wait_bounded(clce_bar(sl), clc_parity(j) ^ 1u, abort_flag, kWaitLimitNs,
                                 kErrTimeoutProducer, &g_device_error_word)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(clcf_bar(sl), 16);
          clc_try_cancel(clc_resp(sl), clcf_bar(sl));
          pending = true;
        }
        const Unit t = unit_at(p, it);
        for (int s = 0; s < t.nsub; ++s) {
          if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, kWaitLimitNs,
                                 kErrTimeoutProducer, &g_device_error_word)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), kStageBytes);
          const uint32_t dst = sbase + kOffA + stage * kStageBytes;
          const int y = t.n0 + s * kSubN;
          tma_load_2d(dst, &tmA, full_bar(stage), t.m0, y);
          tma_load_2d(dst + kHalfBytes, &tmA, full_bar(stage), t.m0 + 64, y);
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        ++k;
        if (p.dynamic) {
          const uint32_t sl = clc_slot(k);
          int nu = -1;
          if (mbar_wait_bounded(clcf_bar(sl), clc_parity(k), abort_flag, kWaitLimitNs,
                                kErrTimeoutProducer, &g_device_error_word)) {
            nu = clc_decode(clc_resp(sl));
            fence_proxy_async_smem();
            mbar_arrive(clce_bar(sl));
            pending = false;
          } else {
            ok = false;
          }
          it.jump(p, nu);
        } else {
          it.next(p);
        }
      }
      if (pending) {
        // A response still on its way lands before the CTA exits.
        volatile uint32_t never = 0u;
        mbar_wait_bounded(clcf_bar(clc_slot(k + 1)), clc_parity(k + 1), &never, kWaitLimitNs,
                          kErrTimeoutDrain, &g_device_error_word);
      }
      if (!ok) {
        // Let the loads already in flight land before the CTA exits.
        volatile uint32_t never_b = 0u;
        if (p.b_tma)
          mbar_wait_bounded(bfull_bar, 0, &never_b, kWaitLimitNs, kErrTimeoutDrain,
                            &g_device_error_word);
        uint32_t st = stage, ph = phase;
        const uint32_t n_pending = issued < (uint32_t)kStages ? issued : (uint32_t)kStages;
        volatile uint32_t never = 0u;
        for (uint32_t i = 0; i < n_pending; ++i) {
          if (st == 0) { st = kStages - 1; ph ^= 1u; } else { --st; }
          mbar_wait_bounded(full_bar(st), ph, &never, kWaitLimitNs, kErrTimeoutDrain,
                            &g_device_error_word);
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------ MMA issuer --------------------------------
    if (lane == 0) {
      const uint64_t bdesc = umma_smem_desc(sbase + kOffB, 256, 128, 0);
      uint32_t stage = 0, phase = 0, acc = 0, accph = 0;
      bool ok = true;
      if (p.b_tma && !mbar_wait_bounded(bfull_bar, 0, abort_flag, kWaitLimitNs, kErrTimeoutMma,
                                        &g_device_error_word))
        ok = false;
      UnitIter it;
      uint32_t k = 0;
      for (it.init(p); it.valid(p) && ok;) {
        const Unit t = unit_at(p, it);
        for (int a = 0; a < t.nacc && ok; ++a) {
          if (!mbar_wait_bounded(acce_bar(acc), accph ^ 1u, abort_flag, kWaitLimitNs,
                                 kErrTimeoutMma, &g_device_error_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nh = (t.nsub - 2 * a) < 2 ? (t.nsub - 2 * a) : 2;
          for (int h = 0; h < nh; ++h) {
            if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, kWaitLimitNs,
                                   kErrTimeoutMma, &g_device_error_word)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = sbase + kOffA + stage * kStageBytes;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              // A: 128 (m) x 16 (k) MN-major, 128-byte swizzle; the two 64-row
              // halves are 8 KiB apart (LBO), 8-column groups 1 KiB apart (SBO).
              const uint64_t adesc = umma_smem_desc(a_base + g * 2048, kHalfBytes, 1024, 2);
              tc_mma_f16_overwrite(tmem_base + acc * kAccN + h * kSubN + g * 16, adesc, bdesc,
                                   kIdesc);
            }
            tc_commit(empty_bar(stage));
            if (++stage == kStages) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          tc_commit(accf_bar(acc));
          if (++acc == kAccStages) { acc = 0; accph ^= 1u; }
        }
        if (!ok) break;
        ++k;
        if (p.dynamic) {
          const uint32_t sl = clc_slot(k);
          int nu = -1;
          if (mbar_wait_bounded(clcf_bar(sl), clc_parity(k), abort_flag, kWaitLimitNs,
                                kErrTimeoutMma, &g_device_error_word)) {
            nu = clc_decode(clc_resp(sl));
            fence_proxy_async_smem();
            mbar_arrive(clce_bar(sl));
          } else {
            ok = false;
          }
          it.jump(p, nu);
        } else {
          it.next(p);
        }
      }
      // All issued MMAs complete before TMEM is released.
      tc_commit(drain_bar);
      volatile uint32_t never = 0u;
      mbar_wait_bounded(drain_bar, 0, &never, kWaitLimitNs, kErrTimeoutDrain,
                        &g_device_error_word);
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ----------------------------------
    const int ew = warp - 2;
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int g = ew >> 2;            // k-block g of each stage: slices 2g, 2g + 1
    const bool leader = (ew == 0 && lane == 0);

    // The launch's global amax (possibly exchanged with the other GPUs; the
    // producer and MMA warps already stream in meanwhile), then the
    // reciprocal scale of every SFC code:
    // min_nanprop(1 / (E4M3^-1(code) * S_dec), FLT_MAX), accurate or rcp.approx.
    if (leader) *s_amax = launch_amax(p, *p.amax, abort_flag, kWaitLimitNs);
    named_bar_sync(2, kEpiThreads);
    const float gamax = *s_amax;
    if (ew * 32 + lane < 256) {
      const uint32_t code = (uint32_t)(ew * 32 + lane);
      const float qs = e4m3_decode(code) * __fdiv_rn(1.0f, global_encode_scale(gamax));
      const float rcp = FM ? rcp_approx_ftz(qs) : __fdiv_rn(1.0f, qs);
      acc_tab[code] = fmin_nan(rcp, 3.402823466e38f);
    }
    if constexpr (SR) {
      // Philox key schedule k_r = seed + r * (0x9E3779B9, 0xBB67AE85), stored
      // as {k0[r], k1[r]} pairs for 16-byte loads of two rounds at a time
      const int tid = ew * 32 + lane;
      if (tid < 10) {
        const uint64_t seed = p.rng != nullptr ? p.rng[0] : 0ull;
        uint32_t* kt = reinterpret_cast<uint32_t*>(smem + kOffKey);
        kt[2 * tid] = (uint32_t)seed + (uint32_t)tid * 0x9E3779B9u;
        kt[2 * tid + 1] = (uint32_t)(seed >> 32) + (uint32_t)tid * 0xBB67AE85u;
      }
    }
    named_bar_sync(2, kEpiThreads);
    const EpiThread e = epi_setup<SR>(p, q, g, lane, sbase + kOffC, sbase + kOffSfc, tmem_base,
                                      sbase + kOffTab, sbase + kOffKey, gamax);

    uint32_t acc = 0, accph = 0, ucount = 0;
    bool ok = true;
    UnitIter it;
    for (it.init(p); it.valid(p); ++ucount) {
      const Unit t = unit_at(p, it);
      const uint32_t buf = ucount & 1u;
      // (ok is true here: a unit after a failed wait ends the walk below)
      ok = epi_cast_unit<SR, FM>(p, t, e, buf, accf_bar(0), acce_bar(0), acc, accph, abort_flag);
      // One barrier per unit among the epilogue warps.  Before it, the leader
      // waits until the previous TMA store has read its staging buffer, which
      // the next unit will overwrite.
      fence_proxy_async_smem();
      if (leader) bulk_wait_read_all();
      if (p.dynamic && ew == 0) {
        // Epilogue warp 0 reads the cluster-launch-control response naming
        // this CTA's next unit, releases the response slot and passes the
        // unit on to the other epilogue warps through shared memory.
        const uint32_t j = ucount + 1, sl = clc_slot(j);
        int nu = -1;
        if (ok && warp_wait(clcf_bar(sl), clc_parity(j), abort_flag, kErrTimeoutEpilogue)) {
          nu = clc_decode(clc_resp(sl));
          fence_proxy_async_smem();
          __syncwarp();
          if (lane == 0) mbar_arrive(clce_bar(sl));
        }
        if (lane == 0) next_unit[buf] = nu;
      }
      __syncwarp();
      named_bar_sync(1, kEpiThreads);
      if (!ok || *abort_flag) {
        ok = false;
        if (p.dynamic) it.jump(p, -1);
        else it.next(p);
        continue;
      }
      epi_store_unit(p, t, &tmC, sbase + kOffC + buf * kCTileBytes,
                     smem + kOffSfc + buf * kSfcTileBytes, ew, lane, leader);
      if (p.dynamic) {
        it.jump(p, next_unit[buf]);
      } else {
        it.next(p);
      }
    }
    if (leader) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Fused amax + cast (one launch): rht_fused_kernel
//
// One CTA per SM (the cooperative launch's co-residency guarantee covers the
// grid barrier) holding two independent pipelines ("halves"), each the same
// producer / MMA / 8-warp epilogue arrangement as rht_nvfp4_kernel with its
// own shared-memory ring, barriers and 256 TMEM columns -- the SM's resources
// are used as by two rht_nvfp4_kernel CTAs.
//   pass 1   the producers stream the tiles of units handed out by a global
//            counter (ascending); the epilogue warps take the NaN-propagating
//            max of |A| straight from the shared-memory stages
//   barrier  the CTAs combine their maxima (and, with world > 1, the ranks')
//   pass 2   the cast, over units handed out in descending order, so that the
//            tiles pass 1 read last are re-read while still in L2; the
//            producer and MMA warps start it before the barrier, only the
//            epilogue needs the amax
// ---------------------------------------------------------------------------
namespace fz {
constexpr int kHalves = 2;
constexpr int kThreadsF = kHalves * kThreads;
constexpr int kQSlots = 4;      // second-pass unit slots per half
// offsets within a half's region
constexpr uint32_t kA = 0;
constexpr uint32_t kC = kA + kStages * kStageBytes;
constexpr uint32_t kSfc = kC + 2 * kCTileBytes;
constexpr uint32_t kEnd = kSfc + 2 * kSfcTileBytes;   // pass-1 end marker, one word per stage
constexpr uint32_t kQ = kEnd + 4 * kStages;            // pass-2 unit slots
constexpr uint32_t kNext = kQ + 4 * kQSlots;           // next unit for the epilogue warps (2 words)
constexpr uint32_t kBar = kNext + 8;
// full, empty, full1, empty1 per stage; accf, acce per accumulator stage;
// drain; qf, qe per unit slot
constexpr uint32_t kNumBarsH = 4 * kStages + 2 * kAccStages + 1 + 2 * kQSlots;
constexpr uint32_t kRegion = ((kBar + 8 * kNumBarsH) + 1023u) & ~1023u;
// shared by the halves
constexpr uint32_t kB = kHalves * kRegion;     // 16 x 16 bf16
constexpr uint32_t kTab = kB + 512;            // 256 reciprocal scales
constexpr uint32_t kKey = kTab + 1024;         // Philox key schedule
constexpr uint32_t kBfull = kKey + 128;        // B's barrier
constexpr uint32_t kMisc = kBfull + 8;         // TMEM base, abort flag, amax
constexpr uint32_t kRed = kMisc + 16;          // per-warp maxima, 16 words
constexpr uint32_t kSmemBytes = kRed + 64 + 1024;   // + alignment slack
static_assert(kSmemBytes <= 227 * 1024, "fused kernel shared memory");
static_assert(kEnd % 16 == 0 && kBar % 8 == 0, "fused kernel layout");
}  // namespace fz

template <bool SR, bool FM>
__global__ void __launch_bounds__(fz::kThreadsF, 1)
    rht_fused_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmC,
                     const __grid_constant__ CUtensorMap tmB, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  const uint32_t sbase = smem_addr(smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int half = warp / (kThreads / 32);
  const int lw = warp - half * (kThreads / 32);   // warp within the half: 0 producer, 1 MMA
  uint8_t* hs = smem + half * fz::kRegion;
  const uint32_t hbase = sbase + half * fz::kRegion;

  const uint32_t bar0 = hbase + fz::kBar;
  auto full_bar = [&](uint32_t s) { return bar0 + 8 * s; };
  auto empty_bar = [&](uint32_t s) { return bar0 + 8 * (kStages + s); };
  auto full1_bar = [&](uint32_t s) { return bar0 + 8 * (2 * kStages + s); };
  auto empty1_bar = [&](uint32_t s) { return bar0 + 8 * (3 * kStages + s); };
  const uint32_t accf0 = bar0 + 8 * (4 * kStages);
  const uint32_t acce0 = accf0 + 8 * kAccStages;
  const uint32_t drain_bar = acce0 + 8 * kAccStages;
  auto qf_bar = [&](uint32_t s) { return drain_bar + 8 * (1 + s); };
  auto qe_bar = [&](uint32_t s) { return drain_bar + 8 * (1 + fz::kQSlots + s); };
  const uint32_t bfull_bar = sbase + fz::kBfull;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(smem + fz::kMisc);
  volatile uint32_t* abort_flag = reinterpret_cast<volatile uint32_t*>(smem + fz::kMisc + 4);
  float* s_amax = reinterpret_cast<float*>(smem + fz::kMisc + 8);
  volatile uint32_t* end_flag = reinterpret_cast<volatile uint32_t*>(hs + fz::kEnd);
  volatile int* qslot = reinterpret_cast<volatile int*>(hs + fz::kQ);
  volatile int* next_unit = reinterpret_cast<volatile int*>(hs + fz::kNext);

  if (lw == 0 && lane == 0) {
    // thread 0 of each half: that half's barriers
    for (uint32_t s = 0; s < kStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
      mbar_init(full1_bar(s), 1);
      mbar_init(empty1_bar(s), kEpiThreads);
    }
    for (uint32_t a = 0; a < kAccStages; ++a) {
      mbar_init(accf0 + 8 * a, 1);
      mbar_init(acce0 + 8 * a, kEpiThreads);
    }
    mbar_init(drain_bar, 1);
    for (uint32_t s = 0; s < (uint32_t)fz::kQSlots; ++s) {
      mbar_init(qf_bar(s), 1);
      mbar_init(qe_bar(s), 2);   // MMA, epilogue warp 0
    }
    if (half == 0) {
      mbar_init(bfull_bar, 1);
      *abort_flag = 0u;
    }
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmC);
    if (p.b_tma) prefetch_tmap(&tmB);
  }
  if (warp == 1) {
    if (!p.b_tma) {
      // B into shared memory in the canonical no-swizzle MN-major layout
      uint16_t* sb = reinterpret_cast<uint16_t*>(smem + fz::kB);
      for (int idx = lane; idx < 256; idx += 32) {
        const int k = idx >> 4, c = idx & 15;
        const uint32_t off = (c & 7) * 2 + (k & 7) * 16 + (c >> 3) * 128 + (k >> 3) * 256;
        sb[off >> 1] = p.B[idx];
      }
      fence_proxy_async_smem();
    }
    tmem_alloc(smem_addr(tmem_holder), fz::kHalves * kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_all = *tmem_holder;
  const uint32_t tmem_base = tmem_all + (uint32_t)half * kTmemCols;
  const uint32_t units = (uint32_t)p.units;

  if (lw == 0) {
    // ------------------------------ TMA producer ------------------------------
    if (lane == 0) {
      // The launch's generation selects its second-pass counter; it is read
      // before this CTA can reach the grid barrier, which advances it.
      const uint32_t gen = ld_acquire_gpu_u32(p.ws + kWsGen);
      bool ok = true;
      if (half == 0 && p.b_tma) {
        mbar_arrive_expect_tx(bfull_bar, 512);
        tma_load_4d(sbase + fz::kB, &tmB, bfull_bar);
      }
      // Pass 1: units from the first counter; after the last, an end marker
      // posted on the next stage.
      uint32_t st = 0, ph = 0, posted = 0;
      uint32_t u_next = atomicAdd(p.ws + kWsCnt1, 1u);
      while (ok) {
        // the unit after this one is requested before this one's loads
        const uint32_t u = u_next;
        const bool last = u >= units;
        if (!last) u_next = atomicAdd(p.ws + kWsCnt1, 1u);
        Unit t;
        t.nsub = 1;
        if (!last) t = unit_of(p, (int)u);
        for (int s = 0; s < t.nsub; ++s) {
          if (!mbar_wait_bounded(empty1_bar(st), ph ^ 1u, abort_flag, kWaitLimitNs,
                                 kErrTimeoutProducer, &g_device_error_word)) {
            ok = false;
            break;
          }
          if (last) {
            end_flag[st] = 1u;
            mbar_arrive(full1_bar(st));
          } else {
            end_flag[st] = 0u;
            mbar_arrive_expect_tx(full1_bar(st), kStageBytes);
            const uint32_t dst = hbase + fz::kA + st * kStageBytes;
            const int y = t.n0 + s * kSubN;
            tma_load_2d(dst, &tmA, full1_bar(st), t.m0, y);
            tma_load_2d(dst + kHalfBytes, &tmA, full1_bar(st), t.m0 + 64, y);
          }
          ++posted;
          if (++st == kStages) { st = 0; ph ^= 1u; }
        }
        if (last) break;
      }
      // Every first-pass posting completes (bounded, whatever happened), and
      // the second pass reuses a stage only after the epilogue has read it.
      {
        const uint32_t pend = posted < (uint32_t)kStages ? posted : (uint32_t)kStages;
        volatile uint32_t never = 0u;
        for (uint32_t i = 0; i < pend; ++i) {
          if (st == 0) { st = kStages - 1; ph ^= 1u; } else { --st; }
          mbar_wait_bounded(full1_bar(st), ph, &never, kWaitLimitNs, kErrTimeoutDrain,
                            &g_device_error_word);
          if (ok && !mbar_wait_bounded(empty1_bar(st), ph, abort_flag, kWaitLimitNs,
                                       kErrTimeoutProducer, &g_device_error_word))
            ok = false;
        }
      }
      // Pass 2: units in descending order, each posted to the MMA and the
      // epilogue one unit ahead of its loads.
      uint32_t* cnt2 = p.ws + kWsCnt2 + (gen & 1u);
      auto fetch = [&]() -> int {
        const uint32_t u = atomicAdd(cnt2, 1u);
        return u < units ? (int)(units - 1u - u) : -1;
      };
      auto post = [&](uint32_t j, int unit) -> bool {
        const uint32_t sl = j % (uint32_t)fz::kQSlots, par = (j / (uint32_t)fz::kQSlots) & 1u;
        if (!mbar_wait_bounded(qe_bar(sl), par ^ 1u, abort_flag, kWaitLimitNs,
                               kErrTimeoutProducer, &g_device_error_word))
          return false;
        qslot[sl] = unit;
        mbar_arrive(qf_bar(sl));
        return true;
      };
      uint32_t stage = 0, phase = 0, issued = 0, j = 0;
      int cur = ok ? fetch() : -1;
      if (!post(0, cur)) ok = false;
      while (ok && cur >= 0) {
        const int nxt = fetch();
        if (!post(j + 1, nxt)) {
          ok = false;
          break;
        }
        const Unit t = unit_of(p, cur);
        for (int s = 0; s < t.nsub; ++s) {
          if (!mbar_wait_bounded(empty_bar(stage), phase ^ 1u, abort_flag, kWaitLimitNs,
                                 kErrTimeoutProducer, &g_device_error_word)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(stage), kStageBytes);
          const uint32_t dst = hbase + fz::kA + stage * kStageBytes;
          const int y = t.n0 + s * kSubN;
          tma_load_2d(dst, &tmA, full_bar(stage), t.m0, y);
          tma_load_2d(dst + kHalfBytes, &tmA, full_bar(stage), t.m0 + 64, y);
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        cur = nxt;
        ++j;
      }
      if (!ok) {
        // Let the loads already in flight land before the CTA exits.
        volatile uint32_t never = 0u;
        if (half == 0 && p.b_tma)
          mbar_wait_bounded(bfull_bar, 0, &never, kWaitLimitNs, kErrTimeoutDrain,
                            &g_device_error_word);
        uint32_t st2 = stage, ph2 = phase;
        const uint32_t n_pending = issued < (uint32_t)kStages ? issued : (uint32_t)kStages;
        for (uint32_t i = 0; i < n_pending; ++i) {
          if (st2 == 0) { st2 = kStages - 1; ph2 ^= 1u; } else { --st2; }
          mbar_wait_bounded(full_bar(st2), ph2, &never, kWaitLimitNs, kErrTimeoutDrain,
                            &g_device_error_word);
        }
      }
    }
    __syncwarp();
  } else if (lw == 1) {
    // ------------------------------ MMA issuer (pass 2) -----------------------
    if (lane == 0) {
      const uint64_t bdesc = umma_smem_desc(sbase + fz::kB, 256, 128, 0);
      uint32_t stage = 0, phase = 0, acc = 0, accph = 0, j = 0;
      bool ok = true;
      if (p.b_tma && !mbar_wait_bounded(bfull_bar, 0, abort_flag, kWaitLimitNs, kErrTimeoutMma,
                                        &g_device_error_word))
        ok = false;
      while (ok) {
        const uint32_t sl = j % (uint32_t)fz::kQSlots, par = (j / (uint32_t)fz::kQSlots) & 1u;
        if (!mbar_wait_bounded(qf_bar(sl), par, abort_flag, kWaitLimitNs, kErrTimeoutMma,
                               &g_device_error_word))
          break;
        const int unit = qslot[sl];
        mbar_arrive(qe_bar(sl));
        ++j;
        if (unit < 0) break;
        const Unit t = unit_of(p, unit);
        for (int a = 0; a < t.nacc && ok; ++a) {
          if (!mbar_wait_bounded(acce0 + 8 * acc, accph ^ 1u, abort_flag, kWaitLimitNs,
                                 kErrTimeoutMma, &g_device_error_word)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const int nh = (t.nsub - 2 * a) < 2 ? (t.nsub - 2 * a) : 2;
          for (int h = 0; h < nh; ++h) {
            if (!mbar_wait_bounded(full_bar(stage), phase, abort_flag, kWaitLimitNs,
                                   kErrTimeoutMma, &g_device_error_word)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const uint32_t a_base = hbase + fz::kA + stage * kStageBytes;
#pragma unroll
            for (int g = 0; g < 4; ++g) {
              const uint64_t adesc = umma_smem_desc(a_base + g * 2048, kHalfBytes, 1024, 2);
              tc_mma_f16_overwrite(tmem_base + acc * kAccN + h * kSubN + g * 16, adesc, bdesc,
                                   kIdesc);
            }
            tc_commit(empty_bar(stage));
            if (++stage == kStages) { stage = 0; phase ^= 1u; }
          }
          if (!ok) break;
          tc_commit(accf0 + 8 * acc);
          if (++acc == kAccStages) { acc = 0; accph ^= 1u; }
        }
      }
      // All issued MMAs complete before TMEM is released.
      tc_commit(drain_bar);
      volatile uint32_t never = 0u;
      mbar_wait_bounded(drain_bar, 0, &never, kWaitLimitNs, kErrTimeoutDrain,
                        &g_device_error_word);
    }
    __syncwarp();
  } else {
    // ------------------------------ epilogue ----------------------------------
    const int ew = lw - 2;
    const int q = warp & 3;           // TMEM lane quarter this warp may access
    const int g = ew >> 2;            // k-block g of each stage: slices 2g, 2g + 1
    const bool leader = (ew == 0 && lane == 0);
    const bool cta_leader = leader && half == 0;
    const uint32_t unit_bar = 1 + (uint32_t)half;   // named barrier of this half's epilogue
    constexpr uint32_t kBothBar = 3;                // both halves' epilogues
    const int tid = ew * 32 + lane;
    uint32_t gen = 0;
    if (cta_leader) gen = ld_acquire_gpu_u32(p.ws + kWsGen);   // before this block arrives

    // Pass 1: NaN-propagating max of |A| (unsigned max of the bf16
    // magnitude bits) over every stage this half's producer posts, 64 bytes
    // per thread per 16 KiB stage, until the end marker.
    uint32_t m2 = 0, st = 0, ph = 0;
    while (true) {
      if (!warp_wait(full1_bar(st), ph, abort_flag, kErrTimeoutEpilogue)) break;
      const bool end = end_flag[st] != 0u;
      if (!end) {
        const uint32_t src = hbase + fz::kA + st * kStageBytes + (uint32_t)tid * 64u;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint4 x = lds128(src + 16 * i);
          m2 = __vmaxu2(m2, x.x & 0x7FFF7FFFu);
          m2 = __vmaxu2(m2, x.y & 0x7FFF7FFFu);
          m2 = __vmaxu2(m2, x.z & 0x7FFF7FFFu);
          m2 = __vmaxu2(m2, x.w & 0x7FFF7FFFu);
        }
      }
      mbar_arrive(empty1_bar(st));
      if (++st == kStages) { st = 0; ph ^= 1u; }
      if (end) break;
    }
    const uint32_t mw = __reduce_max_sync(0xFFFFFFFFu, max(m2 & 0xFFFFu, m2 >> 16));
    uint32_t* red = reinterpret_cast<uint32_t*>(smem + fz::kRed);
    if (lane == 0) red[half * kEpiWarps + ew] = mw;
    named_bar_sync(kBothBar, fz::kHalves * kEpiThreads);
    if (cta_leader) {
      // Grid barrier: each block folds its maximum into this launch's amax
      // word (atomic max on the bits: amax >= 0, so integer order is value
      // order and NaN wins) and arrives; the last to arrive clears the
      // first-pass counter and the next launch's second-pass counter and
      // amax word, and releases the grid.
      uint32_t cta = 0;
      for (int w = 0; w < fz::kHalves * kEpiWarps; ++w) cta = max(cta, red[w]);
      const uint32_t par = gen & 1u;
      atomicMax(p.ws + kWsAmax + par, cta << 16);      // this block's amax as fp32 bits
      if (atom_add_acq_rel_gpu(p.ws + kWsArrive, 1u) == gridDim.x - 1) {
        volatile uint32_t* ws = p.ws;
        ws[kWsArrive] = 0u;
        ws[kWsCnt1] = 0u;
        ws[kWsCnt2 + (par ^ 1u)] = 0u;
        ws[kWsAmax + (par ^ 1u)] = 0u;
        st_release_gpu_u32(p.ws + kWsGen, gen + 1u);   // release the grid
      } else {
        const uint64_t t0 = globaltimer_ns();
        while (ld_acquire_gpu_u32(p.ws + kWsGen) == gen) {
          if (globaltimer_ns() - t0 > kWaitLimitNs || *abort_flag) {
            *abort_flag = 1u;
            atomicCAS(&g_device_error_word, 0u, (uint32_t)kErrTimeoutGridBarrier);
            break;
          }
        }
      }
      const float local = __uint_as_float(ld_acquire_gpu_u32(p.ws + kWsAmax + par));
      const float gm = launch_amax(p, local, abort_flag, kWaitLimitNs);
      if (p.world <= 1 && blockIdx.x == 0 && p.amax_out != nullptr) *p.amax_out = gm;
      *s_amax = gm;
    }
    named_bar_sync(kBothBar, fz::kHalves * kEpiThreads);
    const float gamax = *s_amax;
    if (half == 0) {
      // reciprocal scale of every SFC code, and the Philox key schedule
      const uint32_t code = (uint32_t)tid;
      const float qs = e4m3_decode(code) * __fdiv_rn(1.0f, global_encode_scale(gamax));
      const float rcp = FM ? rcp_approx_ftz(qs) : __fdiv_rn(1.0f, qs);
      reinterpret_cast<float*>(smem + fz::kTab)[code] = fmin_nan(rcp, 3.402823466e38f);
      if (SR && tid < 10) {
        const uint64_t seed = p.rng != nullptr ? p.rng[0] : 0ull;
        uint32_t* kt = reinterpret_cast<uint32_t*>(smem + fz::kKey);
        kt[2 * tid] = (uint32_t)seed + (uint32_t)tid * 0x9E3779B9u;
        kt[2 * tid + 1] = (uint32_t)(seed >> 32) + (uint32_t)tid * 0xBB67AE85u;
      }
    }
    named_bar_sync(kBothBar, fz::kHalves * kEpiThreads);
    const EpiThread e = epi_setup<SR>(p, q, g, lane, hbase + fz::kC, hbase + fz::kSfc, tmem_base,
                                      sbase + fz::kTab, sbase + fz::kKey, gamax);

    // Pass 2: units from this half's slots; epilogue warp 0 reads each slot
    // and passes the unit on through shared memory.
    auto take = [&](uint32_t j, bool ok_in) -> int {
      const uint32_t sl = j % (uint32_t)fz::kQSlots, par = (j / (uint32_t)fz::kQSlots) & 1u;
      int u = -1;
      if (ok_in && warp_wait(qf_bar(sl), par, abort_flag, kErrTimeoutEpilogue)) {
        u = qslot[sl];
        __syncwarp();
        if (lane == 0) mbar_arrive(qe_bar(sl));
      }
      return u;
    };
    bool ok = !*abort_flag;
    if (ew == 0) {
      const int u = take(0, ok);
      if (lane == 0) next_unit[0] = u;
    }
    __syncwarp();
    named_bar_sync(unit_bar, kEpiThreads);
    int cur = next_unit[0];
    uint32_t acc = 0, accph = 0, j = 1;
    while (cur >= 0) {
      const Unit t = unit_of(p, cur);
      const uint32_t buf = j & 1u;
      ok = epi_cast_unit<SR, FM>(p, t, e, buf, accf0, acce0, acc, accph, abort_flag);
      fence_proxy_async_smem();
      if (leader) bulk_wait_read_all();
      if (ew == 0) {
        const int u = take(j, ok);
        if (lane == 0) next_unit[buf] = u;
      }
      __syncwarp();
      named_bar_sync(unit_bar, kEpiThreads);
      // (a warp whose wait gave up set the abort flag before the barrier)
      if (!ok || *abort_flag) break;
      epi_store_unit(p, t, &tmC, hbase + fz::kC + buf * kCTileBytes,
                     hs + fz::kSfc + buf * kSfcTileBytes, ew, lane, leader);
      cur = next_unit[buf];
      ++j;
    }
    if (leader) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_all, fz::kHalves * kTmemCols);
  }
}


// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

struct MapKey {
  uintptr_t ptr;
  uint64_t d0, d1;
  int kind;
  bool operator==(const MapKey& o) const {
    return ptr == o.ptr && d0 == o.d0 && d1 == o.d1 && kind == o.kind;
  }
};
struct MapKeyHash {
  size_t operator()(const MapKey& k) const {
    return std::hash<uintptr_t>()(k.ptr) ^ (std::hash<uint64_t>()(k.d0 * 1315423911u + k.d1) << 1) ^
           (size_t)k.kind;
  }
};

// Encoded tensor maps are cached by (address, shape); encoding costs a few
// microseconds of host time per call otherwise.
int get_tensor_map(int kind, void* ptr, uint64_t d0, uint64_t d1, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<MapKey, CUtensorMap, MapKeyHash> cache;
  const MapKey key{reinterpret_cast<uintptr_t>(ptr), d0, d1, kind};
  {
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) {
      *out = it->second;
      return NVFP4_OK;
    }
  }
  auto fn = encode_fn();
  if (!fn) return cuda_status(cudaErrorNotSupported);
  CUtensorMap map;
  CUresult res;
  const cuuint32_t estride[2] = {1, 1};
  if (kind == 0) {
    // A: bf16, dims {m, n}, box 64 x 64, 128-byte swizzle
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {d0 * 2};
    const cuuint32_t box[2] = {64, 64};
    res = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, ptr, dims, strides, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else if (kind == 2) {
    // B: the row-major 16 x 16 bf16 matrix seen as (c % 8, k % 8, c / 8, k / 8)
    // with byte strides 2, 32, 16, 256; one 8 x 8 x 2 x 2 box lands in shared
    // memory in the canonical no-swizzle MN-major layout of the MMA's B operand.
    const cuuint64_t dims[4] = {8, 8, 2, 2};
    const cuuint64_t strides[3] = {32, 16, 256};
    const cuuint32_t box[4] = {8, 8, 2, 2};
    const cuuint32_t es4[4] = {1, 1, 1, 1};
    res = fn(&map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, ptr, dims, strides, box, es4,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  } else {
    // C: bytes, dims {n/2, m}, box 128 x 128, 128-byte swizzle
    const cuuint64_t dims[2] = {d0, d1};
    const cuuint64_t strides[1] = {d0};
    const cuuint32_t box[2] = {128, 128};
    res = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, ptr, dims, strides, box, estride,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (res != CUDA_SUCCESS) return NVFP4_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lk(mu);
  if (cache.size() > 256) cache.clear();
  cache.emplace(key, map);
  *out = map;
  return NVFP4_OK;
}

// The kernel of a (SR, FM, fused) combination with its launch shape.
template <bool SR, bool FM, bool FUSED>
struct KernelOf {
  static constexpr auto fn = FUSED ? rht_fused_kernel<SR, FM> : rht_nvfp4_kernel<SR, FM>;
  static constexpr int threads = FUSED ? fz::kThreadsF : kThreads;
  static constexpr uint32_t smem = FUSED ? fz::kSmemBytes : kSmemBytes;
};

// Per-device, once: the kernel's shared-memory attributes; for the fused
// kernel also the number of its blocks that fit on one SM (a cooperative
// launch admits no more).
template <bool SR, bool FM, bool FUSED>
int prepare_kernel(int* per_sm) {
  using K = KernelOf<SR, FM, FUSED>;
  static std::atomic<int> attr_set[64];
  static std::atomic<int> occupancy[64];
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return cuda_status(e);
  if (dev >= 64 || !attr_set[dev].load(std::memory_order_acquire)) {
    if (cudaError_t e = cudaFuncSetAttribute(K::fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)K::smem))
      return cuda_status(e);
    // The largest shared-memory carveout: two CTAs of the cast kernel, or
    // the fused kernel's two pipelines, fit on every SM.
    if (cudaError_t e = cudaFuncSetAttribute(K::fn, cudaFuncAttributePreferredSharedMemoryCarveout,
                                             (int)cudaSharedmemCarveoutMaxShared))
      return cuda_status(e);
    if (dev < 64) attr_set[dev].store(1, std::memory_order_release);
  }
  if constexpr (FUSED) {
    int n = dev < 64 ? occupancy[dev].load(std::memory_order_relaxed) : 0;
    if (n <= 0) {
      if (cudaError_t e =
              cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, K::fn, K::threads, K::smem))
        return cuda_status(e);
      if (n < 1) return cuda_status(cudaErrorCooperativeLaunchTooLarge);
      if (dev < 64) occupancy[dev].store(n, std::memory_order_relaxed);
    }
    *per_sm = n;
  } else {
    *per_sm = 2;
  }
  return NVFP4_OK;
}

template <bool SR, bool FM, bool FUSED>
int launch_kernel(const CUtensorMap& ta, const CUtensorMap& tc, const CUtensorMap& tb,
                  const Params& p, int grid, cudaStream_t stream) {
  using K = KernelOf<SR, FM, FUSED>;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(K::threads);
  cfg.dynamicSmemBytes = K::smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  if constexpr (!FUSED) {
    // A programmatic dependent of the previous kernel in the stream: its
    // launch and prologue overlap that kernel's tail.
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
  } else {
    // The fused kernel's blocks meet at a grid barrier: a cooperative launch
    // guarantees they are all resident.
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
  }
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaError_t e = cudaLaunchKernelEx(&cfg, K::fn, ta, tc, tb, p)) return cuda_status(e);
  return cuda_status(cudaGetLastError());
}

struct KernelEntry {
  int (*prepare)(int*);
  int (*launch)(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const Params&, int,
                cudaStream_t);
};
template <bool SR, bool FM, bool FUSED>
constexpr KernelEntry entry_for() {
  return {&prepare_kernel<SR, FM, FUSED>, &launch_kernel<SR, FM, FUSED>};
}
KernelEntry kernel_entry(bool sr, bool fm, bool fused) {
  static constexpr KernelEntry table[8] = {
      entry_for<false, false, false>(), entry_for<false, true, false>(),
      entry_for<true, false, false>(),  entry_for<true, true, false>(),
      entry_for<false, false, true>(),  entry_for<false, true, true>(),
      entry_for<true, false, true>(),   entry_for<true, true, true>()};
  return table[(fused ? 4 : 0) + (sr ? 2 : 0) + (fm ? 1 : 0)];
}

// How the fused kernel's workspace is handled.
enum class WsMode {
  kCaller,      // caller-owned workspace, zeroed by the caller before first use
  kStaticClear  // the library's static scratch: its counters and amax words are
                // cleared (a 24-byte memset on the stream) right before the
                // launch, after every check has passed
};

int rht_launch(int m, int n, const void* A, const void* B, void* C, void* SFC,
               const float* global_amax, const size_t* rng_state, uint32_t sm_count,
               cudaStream_t stream, int k_tile_size, int sr, int fm, int n_offset, int n_total,
               const unsigned long long* const* ex_peers = nullptr, int ex_rank = 0,
               int ex_world = 1, uint32_t ex_epoch = 0, float* amax_out = nullptr,
               uint32_t* fused_ws = nullptr, WsMode ws_mode = WsMode::kCaller) {
  if (m < 0 || n < 0) return NVFP4_ERR_INVALID_SHAPE;
  if (m == 0 || n == 0) return NVFP4_OK;
  if (m % kBM != 0 || n % 64 != 0 || k_tile_size < 64) return NVFP4_ERR_INVALID_SHAPE;
  if (n_total <= 0) n_total = n;
  if (n_offset < 0 || (int64_t)n_offset + n > (int64_t)n_total) return NVFP4_ERR_INVALID_SHAPE;
  const int kt = n_total < k_tile_size ? n_total : k_tile_size;
  const uint32_t ktm = (uint32_t)(kt / 64);
  if (n_offset % (int)(ktm * 64) != 0) return NVFP4_ERR_INVALID_SHAPE;
  const bool fused = fused_ws != nullptr;
  if (!A || !B || !C || !SFC || (!global_amax && !fused)) return NVFP4_ERR_INVALID_ARGUMENT;
  if (fused && (uintptr_t)fused_ws % 4) return NVFP4_ERR_MISALIGNED;
  if ((uintptr_t)A % 16 || (uintptr_t)C % 16 || (uintptr_t)B % 2) return NVFP4_ERR_MISALIGNED;
  // Work units are counted in 32-bit integers (the grid of the balanced
  // schedule, the fused kernel's unit counters): at most 2^31 - 1 of them.
  const int64_t units64 = (int64_t)(m / kBM) * (((int64_t)n + kUnitN - 1) / kUnitN);
  if (units64 > (int64_t)kMaxUnits)
    return ws_mode == WsMode::kStaticClear ? NVFP4_ERR_SCRATCH_CAPACITY : NVFP4_ERR_INVALID_SHAPE;
  int sms = 0;
  if (int e = device_sm_count(&sms)) return e;

  CUtensorMap ta, tc, tb;
  std::memset(&tb, 0, sizeof(tb));
  if (int e = get_tensor_map(0, const_cast<void*>(A), (uint64_t)m, (uint64_t)n, &ta)) return e;
  if (int e = get_tensor_map(1, C, (uint64_t)(n / 2), (uint64_t)m, &tc)) return e;

  Params p;
  p.m = m;
  p.n = n;
  p.tiles_m = m / kBM;
  p.units = (int)units64;
  p.n_offset = n_offset;
  p.ktm = ktm;
  p.div_ktm = make_fast_div(ktm);
  p.div_tiles_m = make_fast_div((uint32_t)p.tiles_m);
  const uintptr_t sfc_addr = reinterpret_cast<uintptr_t>(SFC);
  p.sfc_vec = ((n / 16) % 16 == 0 && sfc_addr % 16 == 0) ? 16 : (sfc_addr % 4 == 0 ? 4 : 1);
  p.B = reinterpret_cast<const uint16_t*>(B);
  p.sfc = reinterpret_cast<uint8_t*>(SFC);
  p.amax = global_amax;
  p.rng = rng_state;
  p.peers = ex_peers;
  p.rank = ex_rank;
  p.world = ex_peers ? ex_world : 1;
  p.epoch = ex_epoch;
  p.amax_out = amax_out;
  p.ws = fused_ws;
  p.dynamic = 0;
  p.b_tma = (reinterpret_cast<uintptr_t>(B) % 16 == 0) ? 1 : 0;
  // (a B whose view the driver will not encode takes the copy path instead)
  if (p.b_tma && get_tensor_map(2, const_cast<void*>(B), 16, 16, &tb) != NVFP4_OK) p.b_tma = 0;

  int grid = sms;
  if (sm_count > 0 && (int)sm_count < grid) grid = (int)sm_count;
  if (fused) {
    // one CTA (two pipelines) per SM, no more than the units can keep busy
    if ((p.units + 1) / 2 < grid) grid = (p.units + 1) / 2;
  } else {
    grid *= 2;   // two CTAs per SM
    if (p.units < grid) grid = p.units;
    if (grid == 2 * sms) {
      // All SMs in use: one CTA per unit, balanced by cluster launch control.
      p.dynamic = 1;
      grid = p.units;
    }
  }

  const KernelEntry k = kernel_entry(sr, fm, fused);
  int per_sm = 0;
  if (int e = k.prepare(&per_sm)) return e;
  if (fused) {
    if (grid > per_sm * sms) grid = per_sm * sms;   // all blocks resident
    if (ws_mode == WsMode::kStaticClear) {
      if (cudaError_t e = cudaMemsetAsync(fused_ws, 0, kWsClearBytes, stream))
        return cuda_status(e);
    }
  }
  return k.launch(ta, tc, tb, p, grid, stream);
}

}  // namespace rht

// ---------------------------------------------------------------------------
// Shared host helpers
// ---------------------------------------------------------------------------
namespace {
thread_local int t_last_cuda_error = 0;
}

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return NVFP4_OK;
  t_last_cuda_error = (int)e;
  return NVFP4_ERR_CUDA;
}

int device_sm_count(int* sms) {
  static std::atomic<int> cache[64];
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return cuda_status(e);
  if (dev < 64) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) {
      *sms = c;
      return NVFP4_OK;
    }
  }
  int major = 0, minor = 0, count = 0;
  if (cudaError_t e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev))
    return cuda_status(e);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  if (major != 10 || minor != 0) return NVFP4_ERR_UNSUPPORTED_DEVICE;
  if (cudaError_t e = cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, dev))
    return cuda_status(e);
  if (dev < 64) cache[dev].store(count, std::memory_order_relaxed);
  *sms = count;
  return NVFP4_OK;
}

}  // namespace nvfp4

using nvfp4::rht::rht_launch;

extern "C" {

NVFP4_API const char* nvfp4_status_string(int status) {
  switch (status) {
    case NVFP4_OK: return "ok";
    case NVFP4_ERR_INVALID_SHAPE: return "invalid shape (m % 128, n % 64, cols % 16 or k_tile_size)";
    case NVFP4_ERR_INVALID_ARGUMENT: return "invalid argument (null pointer or bad flags)";
    case NVFP4_ERR_MISALIGNED: return "misaligned pointer";
    case NVFP4_ERR_CUDA: return "CUDA runtime error";
    case NVFP4_ERR_UNSUPPORTED_DEVICE: return "unsupported device (needs compute capability 10.0)";
    case NVFP4_ERR_DEVICE_TIMEOUT: return "a kernel wait timed out";
    case NVFP4_ERR_SCRATCH_CAPACITY:
      return "problem has more work units (128 x 256 tiles) than the no-allocation entry's "
             "built-in scratch counts (2^31 - 1)";
    default: return "unknown status";
  }
}

NVFP4_API int nvfp4_last_cuda_error(void) { return nvfp4::t_last_cuda_error; }

NVFP4_API int nvfp4_rht_gemm_ntt_w_sfc(int m, int n, const void* A, const void* B, void* C,
                                       void* SFC, const float* global_amax,
                                       const size_t* rng_state, uint32_t sm_count,
                                       nvfp4_stream_t stream, int k_tile_size,
                                       int stochastic_rounding, int use_fast_math) {
  return rht_launch(m, n, A, B, C, SFC, global_amax, rng_state, sm_count, (cudaStream_t)stream,
                    k_tile_size, stochastic_rounding != 0, use_fast_math != 0, 0, n);
}

NVFP4_API int nvfp4_rht_gemm_ntt_w_sfc_sharded(int m, int n, const void* A, const void* B,
                                               void* C, void* SFC, const float* global_amax,
                                               const size_t* rng_state, uint32_t sm_count,
                                               nvfp4_stream_t stream, int k_tile_size,
                                               int stochastic_rounding, int use_fast_math,
                                               int n_offset, int n_total) {
  return rht_launch(m, n, A, B, C, SFC, global_amax, rng_state, sm_count, (cudaStream_t)stream,
                    k_tile_size, stochastic_rounding != 0, use_fast_math != 0, n_offset, n_total);
}

NVFP4_API int nvfp4_run_rht(int m, int n, const void* A, const void* B, void* C, void* SFC,
                            const float* global_amax, const size_t* rng_state, uint32_t sm_count,
                            nvfp4_stream_t stream) {
  return nvfp4_rht_gemm_ntt_w_sfc(m, n, A, B, C, SFC, global_amax, rng_state, sm_count, stream,
                                  2048, 0, 0);
}
NVFP4_API int nvfp4_run_rht_fast(int m, int n, const void* A, const void* B, void* C, void* SFC,
                                 const float* global_amax, const size_t* rng_state,
                                 uint32_t sm_count, nvfp4_stream_t stream) {
  return nvfp4_rht_gemm_ntt_w_sfc(m, n, A, B, C, SFC, global_amax, rng_state, sm_count, stream,
                                  2048, 0, 1);
}
NVFP4_API int nvfp4_run_rht_sr(int m, int n, const void* A, const void* B, void* C, void* SFC,
                               const float* global_amax, const size_t* rng_state,
                               uint32_t sm_count, nvfp4_stream_t stream) {
  return nvfp4_rht_gemm_ntt_w_sfc(m, n, A, B, C, SFC, global_amax, rng_state, sm_count, stream,
                                  2048, 1, 0);
}

NVFP4_API int nvfp4_rht_gemm_ttt(int m, int n, const void* A, const void* B, void* C, void* SFC,
                                 const float* global_amax, const size_t* rng_state,
                                 uint32_t sm_count, nvfp4_stream_t stream, int k_tile_size,
                                 int stochastic_rounding, int use_fast_math) {
  return nvfp4_rht_gemm_ntt_w_sfc(n, m, A, B, C, SFC, global_amax, rng_state, sm_count, stream,
                                  k_tile_size, stochastic_rounding, use_fast_math);
}

// ---------------------------------------------------------------------------
// Cross-GPU amax exchange over peer memory
// ---------------------------------------------------------------------------
struct nvfp4_exchange {
  int rank, world, device;
  unsigned long long* local;          // this rank's 2 x world slots
  void* peer[64];                     // every rank's slot array (self = local)
  unsigned long long** dev_peers;     // the same pointers, in device memory
  uint32_t epoch;
};

NVFP4_API int nvfp4_exchange_create(int rank, int world, nvfp4_exchange** out,
                                    void* ipc_handle_out) {
  if (!out || !ipc_handle_out || world < 2 || world > 64 || rank < 0 || rank >= world)
    return NVFP4_ERR_INVALID_ARGUMENT;
  nvfp4_exchange* ex = new nvfp4_exchange();
  ex->rank = rank;
  ex->world = world;
  ex->epoch = 0;
  cudaError_t e = cudaGetDevice(&ex->device);
  if (!e) e = cudaMalloc(&ex->local, 2 * (size_t)world * sizeof(unsigned long long));
  if (!e) e = cudaMemset(ex->local, 0, 2 * (size_t)world * sizeof(unsigned long long));
  if (!e) e = cudaMalloc(&ex->dev_peers, (size_t)world * sizeof(void*));
  if (!e) e = cudaIpcGetMemHandle(reinterpret_cast<cudaIpcMemHandle_t*>(ipc_handle_out), ex->local);
  if (!e) e = cudaDeviceSynchronize();
  if (e) {
    if (ex->local) cudaFree(ex->local);
    if (ex->dev_peers) cudaFree(ex->dev_peers);
    delete ex;
    return nvfp4::cuda_status(e);
  }
  for (int q = 0; q < 64; ++q) ex->peer[q] = nullptr;
  *out = ex;
  return NVFP4_OK;
}

NVFP4_API int nvfp4_exchange_connect(nvfp4_exchange* ex, const void* all_handles) {
  if (!ex || !all_handles) return NVFP4_ERR_INVALID_ARGUMENT;
  const cudaIpcMemHandle_t* h = reinterpret_cast<const cudaIpcMemHandle_t*>(all_handles);
  for (int q = 0; q < ex->world; ++q) {
    if (q == ex->rank) {
      ex->peer[q] = ex->local;
      continue;
    }
    if (cudaError_t e = cudaIpcOpenMemHandle(&ex->peer[q], h[q], cudaIpcMemLazyEnablePeerAccess))
      return nvfp4::cuda_status(e);
  }
  if (cudaError_t e = cudaMemcpy(ex->dev_peers, ex->peer, (size_t)ex->world * sizeof(void*),
                                 cudaMemcpyHostToDevice))
    return nvfp4::cuda_status(e);
  return NVFP4_OK;
}

NVFP4_API int nvfp4_exchange_destroy(nvfp4_exchange* ex) {
  if (!ex) return NVFP4_OK;
  cudaDeviceSynchronize();
  for (int q = 0; q < ex->world; ++q)
    if (q != ex->rank && ex->peer[q]) cudaIpcCloseMemHandle(ex->peer[q]);
  cudaFree(ex->dev_peers);
  cudaFree(ex->local);
  delete ex;
  return NVFP4_OK;
}

NVFP4_API int nvfp4_rht_gemm_ntt_w_sfc_sharded_exchange(
    int m, int n, const void* A, const void* B, void* C, void* SFC, const float* local_amax,
    float* global_amax_out, const size_t* rng_state, uint32_t sm_count, nvfp4_stream_t stream,
    int k_tile_size, int stochastic_rounding, int use_fast_math, int n_offset, int n_total,
    nvfp4_exchange* ex) {
  if (!ex || ex->peer[ex->rank] == nullptr) return NVFP4_ERR_INVALID_ARGUMENT;
  if (m == 0 || n == 0) return NVFP4_ERR_INVALID_SHAPE;   // every rank must join the exchange
  const uint32_t epoch = ex->epoch + 1;   // epochs start at 1: zeroed slots never match
  const int rc = rht_launch(m, n, A, B, C, SFC, local_amax, rng_state, sm_count,
                            (cudaStream_t)stream, k_tile_size, stochastic_rounding != 0,
                            use_fast_math != 0, n_offset, n_total,
                            const_cast<const unsigned long long* const*>(ex->dev_peers), ex->rank,
                            ex->world, epoch, global_amax_out);
  if (rc == NVFP4_OK) ex->epoch = epoch;
  return rc;
}

NVFP4_API size_t nvfp4_fused_workspace_bytes(void) {
  return (size_t)nvfp4::rht::kFusedWsWords * sizeof(uint32_t);
}

NVFP4_API int nvfp4_quantize_rht_fused(int m, int n, const void* A, const void* B, void* C,
                                       void* SFC, float* amax_out, const size_t* rng_state,
                                       uint32_t sm_count, nvfp4_stream_t stream, int k_tile_size,
                                       int stochastic_rounding, int use_fast_math,
                                       void* workspace) {
  if (!workspace) return NVFP4_ERR_INVALID_ARGUMENT;
  return rht_launch(m, n, A, B, C, SFC, nullptr, rng_state, sm_count, (cudaStream_t)stream,
                    k_tile_size, stochastic_rounding != 0, use_fast_math != 0, 0, n, nullptr, 0,
                    1, 0, amax_out, reinterpret_cast<uint32_t*>(workspace));
}

// ---------------------------------------------------------------------------
// Fused amax + cast without any allocation by the caller or the library.
// The workspace (grid-barrier count, unit counters, amax words: kFusedWsWords
// 32-bit words, 32 bytes whatever the problem size) lives in this static
// device array, on every GPU that loads the library, until the process
// exits.  Host code must not hand the array's name to a kernel:
// there it only stands for the symbol, so its device address is looked up
// once per device with cudaGetSymbolAddress.
// ---------------------------------------------------------------------------
namespace {
static __device__ __align__(256) uint32_t g_fused_scratch[nvfp4::rht::kFusedWsWords];

// Device address of g_fused_scratch on the current device, looked up on the
// first call per device and kept.  A cudaDeviceReset unloads the module and
// may move the array, so the kept address is not valid across a reset of a
// device this library has used.
int fused_scratch_address(uint32_t** out) {
  static std::mutex mu;
  static uint32_t* addr[64] = {nullptr};
  int dev = 0;
  if (cudaError_t e = cudaGetDevice(&dev)) return nvfp4::cuda_status(e);
  if (dev >= 64) return NVFP4_ERR_UNSUPPORTED_DEVICE;
  std::lock_guard<std::mutex> lk(mu);
  if (addr[dev] == nullptr) {
    void* ptr = nullptr;
    if (cudaError_t e = cudaGetSymbolAddress(&ptr, g_fused_scratch)) return nvfp4::cuda_status(e);
    addr[dev] = reinterpret_cast<uint32_t*>(ptr);
  }
  *out = addr[dev];
  return NVFP4_OK;
}
}  // namespace

NVFP4_API int nvfp4_quantize_rht_fused_noalloc(int m, int n, const void* A, const void* B,
                                               void* C, void* SFC, float* amax_out,
                                               const size_t* rng_state, uint32_t sm_count,
                                               nvfp4_stream_t stream, int k_tile_size,
                                               int stochastic_rounding, int use_fast_math) {
  // Argument checks that need no device come first (rht_launch repeats them).
  if (m < 0 || n < 0) return NVFP4_ERR_INVALID_SHAPE;
  if (m == 0 || n == 0) return NVFP4_OK;
  if (m % nvfp4::rht::kBM != 0 || n % 64 != 0 || k_tile_size < 64) return NVFP4_ERR_INVALID_SHAPE;
  if (!A || !B || !C || !SFC) return NVFP4_ERR_INVALID_ARGUMENT;
  if ((int64_t)(m / nvfp4::rht::kBM) * (((int64_t)n + nvfp4::rht::kUnitN - 1) / nvfp4::rht::kUnitN) >
      (int64_t)nvfp4::rht::kMaxUnits)
    return NVFP4_ERR_SCRATCH_CAPACITY;
  uint32_t* scratch = nullptr;
  if (int e = fused_scratch_address(&scratch)) return e;
  // rht_launch checks shapes, pointers and the unit count against the
  // scratch's 32-bit counters first; only a call that passes every check
  // enqueues anything: a 24-byte memset of the counters and amax words (a
  // launch that gave up part-way may have left them nonzero), then the kernel.
  return rht_launch(m, n, A, B, C, SFC, nullptr, rng_state, sm_count, (cudaStream_t)stream,
                    k_tile_size, stochastic_rounding != 0, use_fast_math != 0, 0, n, nullptr, 0,
                    1, 0, amax_out, scratch, nvfp4::rht::WsMode::kStaticClear);
}

NVFP4_API int nvfp4_quantize_rht_fused_sharded_exchange(
    int m, int n, const void* A, const void* B, void* C, void* SFC, float* amax_out,
    const size_t* rng_state, uint32_t sm_count, nvfp4_stream_t stream, int k_tile_size,
    int stochastic_rounding, int use_fast_math, int n_offset, int n_total, nvfp4_exchange* ex,
    void* workspace) {
  if (!ex || ex->peer[ex->rank] == nullptr || !workspace) return NVFP4_ERR_INVALID_ARGUMENT;
  if (m == 0 || n == 0) return NVFP4_ERR_INVALID_SHAPE;   // every rank must join the exchange
  const uint32_t epoch = ex->epoch + 1;
  const int rc = rht_launch(m, n, A, B, C, SFC, nullptr, rng_state, sm_count,
                            (cudaStream_t)stream, k_tile_size, stochastic_rounding != 0,
                            use_fast_math != 0, n_offset, n_total,
                            const_cast<const unsigned long long* const*>(ex->dev_peers), ex->rank,
                            ex->world, epoch, amax_out, reinterpret_cast<uint32_t*>(workspace));
  if (rc == NVFP4_OK) ex->epoch = epoch;
  return rc;
}

NVFP4_API int nvfp4_device_error(uint32_t* code, int clear) {
  if (!code) return NVFP4_ERR_INVALID_ARGUMENT;
  if (cudaError_t e = cudaDeviceSynchronize()) return nvfp4::cuda_status(e);
  if (cudaError_t e = cudaMemcpyFromSymbol(code, nvfp4::g_device_error_word, sizeof(uint32_t)))
    return nvfp4::cuda_status(e);
  if (clear) {
    const uint32_t zero = 0;
    if (cudaError_t e = cudaMemcpyToSymbol(nvfp4::g_device_error_word, &zero, sizeof(uint32_t)))
      return nvfp4::cuda_status(e);
  }
  return NVFP4_OK;
}

}  // extern "C"
