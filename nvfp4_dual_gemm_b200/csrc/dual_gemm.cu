// dual_gemm.cu — B200 (sm_100a) NVFP4 dual GEMM  C = silu(A B1^T) * (A B2^T)
//
// One persistent, warp-specialised kernel per tile width BN (64 or 128
// columns of each GEMM); warp roles are described above dual_gemm_kernel.
// Per 256-wide K block the producers stream the A tile (128 x 128 B), the B1
// and B2 tiles (BN x 128 B each, stacked into one 2*BN-row operand) and the
// three 2 KiB block-scale runs through a ring of shared-memory stages; the
// MMA thread issues four tcgen05.mma kind::mxf4nvf4 block_scale (M = 128,
// N = 2*BN, K = 64) into one TMEM accumulator whose columns [0, BN) hold
// A B1^T and [BN, 2*BN) hold A B2^T; the epilogue computes silu(x) * y in
// fp32 and stores fp16 rows, or, for tiles split along K, hands fp32
// partials through the workspace to the last segment to finish.
// The reference kernel is non-persistent with one tile per CTA and issues
// the scale copies and two MMAs per K step from one thread
// (nvfp4_dual_gemm.cu:77-317); the scheduling here is in schedule.h.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <type_traits>
#include <vector>
#include <mutex>
#include <string>
#include <utility>

#include "nvfp4_dual_gemm.h"
#include "schedule.h"
#include "sm100_ptx.cuh"

namespace nvfp4dg {

constexpr int kBM = 128;            // tile rows (TMEM lanes)
constexpr int kRowBytes = 128;      // one stage = 256 fp4 of K = 128 bytes/row
constexpr int kSfAtomBytes = 512;   // 128 rows x 4 scales
constexpr int kSfRunBytes = 2048;   // 4 atoms = the scales of 256 K elements
constexpr int kCBoxBytes = 16384;   // fp16 C store box: 128 rows x 64 columns
constexpr int kThreads = 352;
constexpr int kTmemCols = 512;
constexpr int kSfTmemBase = 256;    // scale regions follow the accumulator
constexpr int kSfTmemPerStage = 48; // SFA 4 x 4 cols, SFB 4 x (4 + 4) cols

// Wait limit of the stream-K owner under NVFP4DG_FLAG_TEST_SK_TIMEOUT
// (~0.5 ms): long enough for every real contribution to land, short enough
// for a test.
constexpr long long kTestWaitLimitCycles = 1000ll * 1000ll;

// Device error word bits (role whose bounded wait expired).
constexpr unsigned kErrProducer = 1u << 0;
constexpr unsigned kErrMma = 1u << 1;
constexpr unsigned kErrEpilogue = 1u << 2;
constexpr unsigned kErrDrain = 1u << 3;

template <int BN>
struct Cfg {
  static constexpr int kStages = (BN == 128) ? 4 : 5;
  static constexpr int kABytes = kBM * kRowBytes;
  static constexpr int kBBytes = BN * kRowBytes;
  static constexpr int kStageBytes = kABytes + 2 * kBBytes + 3 * kSfRunBytes;
  static constexpr int kSmemBytes = kStages * kStageBytes + 1024;
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-B aligned");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert(kSfTmemBase + kStages * kSfTmemPerStage <= kTmemCols,
                "TMEM budget");
  static_assert(2 * BN <= kSfTmemBase, "accumulator must fit below scales");
  static_assert(kStages * kStageBytes >= 4 * 32768,
                "stream-K fixup staging reuses the stage buffers");
};

// Grouped problems (nvfp4_dual_gemm_run_grouped): `count` problems sharing N
// and K whose activations (rows of A, SFA, C) are concatenated, group g at
// rows [row0[g], row0[g] + rows[g]) with row0[g] a multiple of 128, and whose
// weights are batches g of B1 / B2 / SFB1 / SFB2.  Linear tiles [tile0[g],
// tile0[g + 1]) belong to group g (m fastest, as for one problem).
constexpr int kMaxGroups = 64;
struct GroupTable {
  int count;  // 0: not a grouped launch
  int tile0[kMaxGroups + 1];
  int row0[kMaxGroups];
  int rows[kMaxGroups];
};

struct KParams {
  Plan plan;
  int M, N, K;
  // batch l of a batched problem (plan.L > 1): its blocked scales start
  // l * sfa_batch / l * sfb_batch bytes into SFA / SFB1 / SFB2, its rows of
  // C (or of Cq / SFC) l * M * N elements (l * M * N/2 / l * sfc_batch
  // bytes) into C (Cq / SFC); A, B1, B2 are addressed by the tensor maps'
  // third coordinate
  long long sfa_batch, sfb_batch, sfc_batch;
  const uint8_t* sfa;
  const uint8_t* sfb1;
  const uint8_t* sfb2;
  __half* C;
  // NVFP4 output (nvfp4_dual_gemm_run_nvfp4_out): when cq is not null, C is
  // not written; instead each 16-column block of a row of fp16(silu * y) is
  // quantised to e2m1 codes (cq, [M, N/2]) and one e4m3 scale in the
  // blocked layout (sfc, ceil(M/128) * (N/64) * 512 bytes)
  uint8_t* cq;
  uint8_t* sfc;
  float* partials;
  int* counters;
  unsigned* err;
  // 1-SM kernel: tmB1 is a 3-D map whose third coordinate selects B1 (0) or
  // B2 (1), so one copy brings both tiles of a K block (see b_pair_map)
  int b_merged;
  // NVFP4DG_FLAG_STATIC_WEIGHTS: the weight producer (warp 5: B1/B2 tiles and
  // all B scale runs) starts before the dependency wait; the activation
  // producer (warp 4: A and its scales) still waits
  int static_weights;
  // pair kernel: 3-D tensor maps (batch / group coordinate) instead of 2-D
  int maps3d;
  // stream-K owners wait for b_last - b_first + sk_extra contributions, at
  // most sk_wait_limit cycles (sk_extra = 1 and a short limit only under
  // NVFP4DG_FLAG_TEST_SK_TIMEOUT, to make that bounded wait run out)
  int sk_extra;
  long long sk_wait_limit;
  // pair kernel, BN = 128, fp16 C of ungrouped problems (unless
  // NVFP4DG_FLAG_NO_TMA_STORE): whole tiles stage their fp16 outputs in
  // shared memory and store them with TMA through the C tensor map (3-D,
  // the batch as third coordinate, when c_layers > 1)
  int c_tma;
  int c_layers;
  GroupTable groups;
};

__device__ unsigned g_err_word;

// Scratch of nvfp4_dual_gemm_run_noalloc: the stream-K counters and fp32
// partials of one call, for callers that cannot allocate device memory.  In
// host code this name is only a stand-in for the symbol; the device address
// comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char
    g_noalloc_scratch[NVFP4DG_NOALLOC_SCRATCH_BYTES];

// Optional pipeline trace (compile with -DNVFP4DG_TRACE): per CTA, the SM
// clock at each hand-off of the first kTraceSlots main-loop iterations —
// producer after its empty-slot wait (0) and after issuing the copies (1),
// MMA issuer after its full-slot wait (2) and after its commit (3), scale
// warp after its data wait (6) and after its arrival (7) — and per work
// unit the epilogue's accumulator-ready (4) and done (5) times.
#ifdef NVFP4DG_TRACE
constexpr int kTraceSlots = 64;
constexpr int kTraceRoles = 10;
constexpr int kTraceCtas = 160;
__device__ long long g_trace[kTraceCtas][kTraceRoles][kTraceSlots];
#define NVFP4DG_STAMP(role, idx)                                   \
  do {                                                             \
    if (blockIdx.x < kTraceCtas && (idx) < kTraceSlots)            \
      g_trace[blockIdx.x][role][idx] = clock_cycles();             \
  } while (0)
// Global-timer (ns, comparable across SMs) stamps of thread 0 in role 5,
// slots 61-63: kernel entry, end of the prologue, exit (pair kernel also
// 50-52: teardown start, C store boxes read, past the final cluster
// barrier; 53: producer A past the dependency wait); the SM clock at the
// same moments goes to role 4, same slots.
#define NVFP4DG_STAMP_NS(idx)                                      \
  do {                                                             \
    if (threadIdx.x == 0 && blockIdx.x < kTraceCtas) {             \
      long long t_;                                                \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));       \
      g_trace[blockIdx.x][4][idx] = clock_cycles();                \
      g_trace[blockIdx.x][5][idx] = t_;                            \
    }                                                              \
  } while (0)
// The same from whichever thread executes it.
#define NVFP4DG_STAMP_NS_ANY(idx)                                  \
  do {                                                             \
    if (blockIdx.x < kTraceCtas) {                                 \
      long long t_;                                                \
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));       \
      g_trace[blockIdx.x][4][idx] = clock_cycles();                \
      g_trace[blockIdx.x][5][idx] = t_;                            \
    }                                                              \
  } while (0)
#else
#define NVFP4DG_STAMP_NS_ANY(idx) \
  do {                            \
  } while (0)
#define NVFP4DG_STAMP(role, idx) \
  do {                           \
  } while (0)
#define NVFP4DG_STAMP_NS(idx) \
  do {                        \
  } while (0)
#endif

__device__ __forceinline__ void epi_bar() {
  asm volatile("bar.sync 1, 128;" ::: "memory");
}

// Start-up barriers: the producer warps (4, 5) meet warp 0 once it has
// initialised the mbarriers (kBarInit: warp 0 arrives, the producers wait),
// and every other warp meets the others once TMEM is allocated (kBarStart);
// the producers never wait for the TMEM allocation.
constexpr int kBarInit = 5;
constexpr int kBarStart = 6;
__device__ __forceinline__ void named_bar_sync(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}
__device__ __forceinline__ void named_bar_arrive(int id, int n) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Barrier `ID` over 128 threads (four warps) that also ANDs a predicate:
// every thread gets the same answer, so a group that must later meet at the
// same named barrier either continues together or leaves together.
template <int ID>
__device__ __forceinline__ bool group_all(bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred)), "n"(ID)
      : "memory");
  return out != 0;
}

// Start-up barrier initialisation by one warp, one barrier per lane (an
// mbarrier.init is a shared-memory store: 32 lanes do 32 of them in one
// instruction, where one thread would do them one after another): lanes
// [0, S) take full[s], [S, 2S) sfdata[s], [2S, 3S) empty[s], then acc_full,
// acc_empty, drain, ready, the four stream-K fixup barriers and the NRECV
// split-K receive barriers.  Each lane fences its own initialisation; lanes
// [0, S) then arm the first fill of their stage's scale barrier with
// `sf_bytes`.
template <int S, int NRECV>
__device__ __forceinline__ void init_barriers_by_lane(
    int lane, uint64_t* full, uint32_t full_count, uint64_t* sfdata,
    uint64_t* empty, uint64_t* acc_full, uint64_t* acc_empty,
    uint32_t acc_empty_count, uint64_t* drain, uint64_t* ready,
    uint64_t* fix, uint64_t* recv, uint32_t sf_bytes) {
  static_assert(3 * S + 4 + 4 + NRECV <= 32, "one barrier per lane");
  uint64_t* bar = nullptr;
  uint32_t count = 1;
  if (lane < S) {
    bar = full + lane;
    count = full_count;
  } else if (lane < 2 * S) {
    bar = sfdata + (lane - S);
  } else if (lane < 3 * S) {
    bar = empty + (lane - 2 * S);
  } else if (lane == 3 * S) {
    bar = acc_full;
  } else if (lane == 3 * S + 1) {
    bar = acc_empty;
    count = acc_empty_count;
  } else if (lane == 3 * S + 2) {
    bar = drain;
  } else if (lane == 3 * S + 3) {
    bar = ready;
  } else if (lane < 3 * S + 4 + 4) {
    bar = fix + (lane - (3 * S + 4));
  } else if (lane < 3 * S + 8 + NRECV) {
    bar = recv + (lane - (3 * S + 8));
  }
  if (bar != nullptr) {
    mbar_init(bar, count);
    fence_mbar_init();
  }
  if (lane == 0) s_wait_failed = 0u;
  __syncwarp();
  // arm the first scale fill of every stage (bytes may land before or after
  // an arming: a barrier's transaction count may go negative meanwhile)
  if (lane < S) mbar_arrive_expect_tx(sfdata + lane, sf_bytes);
  fence_proxy_async_smem();
}

// silu(x) * y = x * y / (1 + e^-x) for two columns, rounded to fp16 and
// packed (x0 / y0 in the low half).  One special-function (MUFU) operation
// per output: e = 2^(-x log2 e) with ex2.approx; the reciprocal of
// d = 1 + e is computed on the FMA pipe, two outputs per instruction
// (fma.rn.f32x2), by three Newton-Raphson steps r <- r + r (1 - d r) from a
// first guess read off the bits of d (the integer 0x7EF311C3 - bits(d)
// approximates 1/d within 11 % for every positive normal d; here formed from
// -d as 0xFEF311C3 - bits(-d)).  The error is quadratic per step, so after
// three steps the reciprocal is exact to fp32 rounding; the result's
// relative error stays below 4e-6 (from rounding x log2 e, as with any
// exp2-based exp) against the 1e-3 tolerance of the fp16 output.  With
// __expf and __fdividef (two MUFU operations per output) the epilogue was
// bound by the SM's 16 MUFU results per cycle.  The exponent is clamped at
// 126 so that d stays finite: silu(x) for x < -87 is below fp16's range
// either way.
__device__ __forceinline__ uint32_t silu_mul_h2(float x0, float x1, float y0,
                                                float y1) {
  uint32_t h;
  asm("{\n\t"
      ".reg .b64 X, Y, T, ND, R, E, ONE, NL2E;\n\t"
      ".reg .b32 t0, t1, e0, e1, n0, n1, r0, r1;\n\t"
      "mov.b64 X, {%1, %2};\n\t"
      "mov.b64 Y, {%3, %4};\n\t"
      "mov.b64 NL2E, {0xBFB8AA3B, 0xBFB8AA3B};\n\t"  // -log2(e)
      "mov.b64 ONE, {0x3F800000, 0x3F800000};\n\t"
      "mul.rn.f32x2 T, X, NL2E;\n\t"
      "mov.b64 {t0, t1}, T;\n\t"
      "min.f32 t0, t0, 0f42FC0000;\n\t"  // 126
      "min.f32 t1, t1, 0f42FC0000;\n\t"
      "ex2.approx.ftz.f32 e0, t0;\n\t"
      "ex2.approx.ftz.f32 e1, t1;\n\t"
      "sub.rn.f32 n0, 0fBF800000, e0;\n\t"  // -d = -(1 + e)
      "sub.rn.f32 n1, 0fBF800000, e1;\n\t"
      "sub.u32 r0, 0xFEF311C3, n0;\n\t"     // first guess of 1/d
      "sub.u32 r1, 0xFEF311C3, n1;\n\t"
      "mov.b64 ND, {n0, n1};\n\t"
      "mov.b64 R, {r0, r1};\n\t"
      "fma.rn.f32x2 E, ND, R, ONE;\n\t"
      "fma.rn.f32x2 R, R, E, R;\n\t"
      "fma.rn.f32x2 E, ND, R, ONE;\n\t"
      "fma.rn.f32x2 R, R, E, R;\n\t"
      "fma.rn.f32x2 E, ND, R, ONE;\n\t"
      "fma.rn.f32x2 R, R, E, R;\n\t"
      "mul.rn.f32x2 T, X, Y;\n\t"
      "mul.rn.f32x2 T, T, R;\n\t"
      "mov.b64 {r0, r1}, T;\n\t"
      "cvt.rn.f16x2.f32 %0, r1, r0;\n\t"
      "}"
      : "=r"(h)
      : "r"(__float_as_uint(x0)), "r"(__float_as_uint(x1)),
        "r"(__float_as_uint(y0)), "r"(__float_as_uint(y1)));
  return h;
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// One 16-element block -> NVFP4: returns the e4m3 scale byte
// e4m3(amax / 6) (round to nearest even, saturating at 448) and sets w0/w1
// to the eight bytes of e2m1 codes of q = RN(v / scale) rounded to the e2m1
// grid (nearest, ties to the even code, saturating at 6, sign kept), all-zero
// codes when the scale is 0.  The forms below (the compare form for 16-bit
// values, encode_rcp16) give the same codes, so the fused NVFP4 output
// equals quantising the fp16 result, whichever form each side uses.
//
// No division: the e2m1 code of q only depends on how q compares with the
// grid midpoints t in {0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5}, and
// RN(v / s) < t  <=>  v < t * s  (and = <=> =) for every fp32 v and e4m3
// scale s.  t * s has at most 7 significant bits, so it is exact; and with
// s = b 2^e, 1 <= b < 2, t = a 2^f, 1 <= a < 2, the fp32 neighbours of
// t * s lie more than s * ulp(t) / 2 away from it (their spacing is at least
// 2^(e+f-23) > b 2^(e+f-24)), so no v other than t * s has a quotient that
// rounds onto t.  Ties at 0.25, 1.25, 2.5, 5 go down (strict >), those at
// 0.75, 1.75, 3.5 up (>=, written as > the float just below).  With an
// IEEE division per element instead, the NVFP4-output epilogue took 18.5
// instead of 15.2 us on the 256 x 4096 x 7168 problem.
__device__ __forceinline__ uint8_t quant_block16(const float* v, uint32_t& w0,
                                                 uint32_t& w1) {
  float amax = 0.f;
#pragma unroll
  for (int q = 0; q < 16; ++q) amax = fmaxf(amax, fabsf(v[q]));
  const __nv_fp8_storage_t sb =
      __nv_cvt_float_to_fp8(amax / 6.0f, __NV_SATFINITE, __NV_E4M3);
  const float sd =
      __half2float(__half(__nv_cvt_fp8_to_halfraw(sb, __NV_E4M3)));
  w0 = 0;
  w1 = 0;
  if (sd > 0.f) {
    auto below = [](float x) { return __uint_as_float(__float_as_uint(x) - 1u); };
    const float t0 = 0.25f * sd, t1 = below(0.75f * sd), t2 = 1.25f * sd,
                t3 = below(1.75f * sd), t4 = 2.5f * sd, t5 = below(3.5f * sd),
                t6 = 5.0f * sd;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      // the number of midpoints below |v| (t0 < t1 < ... < t6), by a
      // three-level binary search
      const float a = fabsf(v[i]);
      const bool b2 = a > t3;
      const bool b1 = a > (b2 ? t5 : t1);
      const bool b0 = a > (b2 ? (b1 ? t6 : t4) : (b1 ? t2 : t0));
      const uint32_t m = (b2 ? 4u : 0u) | (b1 ? 2u : 0u) | (b0 ? 1u : 0u);
      const uint32_t code = m | ((__float_as_uint(v[i]) >> 28) & 8u);
      if (i < 8)
        w0 |= code << (4 * i);
      else
        w1 |= code << (4 * (i - 8));
    }
  }
  return static_cast<uint8_t>(sb);
}

// The same block quantiser for 16-bit elements (fp16 or bf16), held as
// eight packed pairs (element 2i in the low half of p[i]), two elements per
// instruction.  Every midpoint product t * s (at most 7 significant bits,
// between 2^-11 and 2240) is exact in fp16 and in bf16, and for a 16-bit v,
// v >= T <=> v > the 16-bit value below T; so comparing 16-bit keys with
// packed 2-wide compares gives exactly the codes of the fp32 form above.
// The NVFP4-output epilogue uses this compare form (which keeps the GEMM
// kernels' register allocation as it is); the activation quantiser uses
// quant_block16_x2 below, which gives the same codes with fewer
// instructions and hands blocks holding a NaN to this form.
template <typename H2>
struct Half2Ops;
template <>
struct Half2Ops<__half2> {
  static __device__ __forceinline__ uint32_t bits(float x) {  // x exact
    return __half_as_ushort(__float2half_rn(x));
  }
  static __device__ __forceinline__ float lo(uint32_t u) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(u)));
  }
  static __device__ __forceinline__ float hi(uint32_t u) { return lo(u >> 16); }
  static constexpr uint32_t kInfKey = 0x7C00u;  // |v| bits of +inf
};
template <>
struct Half2Ops<__nv_bfloat162> {
  static __device__ __forceinline__ uint32_t bits(float x) {  // x exact
    return __bfloat16_as_ushort(__float2bfloat16_rn(x));
  }
  static __device__ __forceinline__ float lo(uint32_t u) {
    return __uint_as_float(u << 16);
  }
  static __device__ __forceinline__ float hi(uint32_t u) {
    return __uint_as_float(u & 0xFFFF0000u);
  }
  static constexpr uint32_t kInfKey = 0x7F80u;
};

template <typename H2>
__device__ __forceinline__ H2 as_h2(uint32_t u) {
  return *reinterpret_cast<const H2*>(&u);
}

template <typename H2>
__device__ __forceinline__ uint8_t quant_block16_x2_cmp(const uint32_t (&p)[8],
                                                        uint32_t& w0,
                                                        uint32_t& w1) {
  using Ops = Half2Ops<H2>;
  uint32_t a[8];  // |v| pairs: the keys
#pragma unroll
  for (int i = 0; i < 8; ++i) a[i] = p[i] & 0x7FFF7FFFu;
  H2 m2 = as_h2<H2>(a[0]);
#pragma unroll
  for (int i = 1; i < 8; ++i) m2 = __hmax2(m2, as_h2<H2>(a[i]));
  uint32_t mu;
  *reinterpret_cast<H2*>(&mu) = m2;
  const float amax = fmaxf(Ops::lo(mu), Ops::hi(mu));
  const __nv_fp8_storage_t sb =
      __nv_cvt_float_to_fp8(amax / 6.0f, __NV_SATFINITE, __NV_E4M3);
  const float sd =
      __half2float(__half(__nv_cvt_fp8_to_halfraw(sb, __NV_E4M3)));
  w0 = 0;
  w1 = 0;
  if (sd > 0.f) {
    auto rep2 = [](uint32_t b) { return b | (b << 16); };
    const uint32_t t0 = rep2(Ops::bits(0.25f * sd)),
                   t1 = rep2(Ops::bits(0.75f * sd) - 1u),
                   t2 = rep2(Ops::bits(1.25f * sd)),
                   t3 = rep2(Ops::bits(1.75f * sd) - 1u),
                   t4 = rep2(Ops::bits(2.5f * sd)),
                   t5 = rep2(Ops::bits(3.5f * sd) - 1u),
                   t6 = rep2(Ops::bits(5.0f * sd));
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const H2 k = as_h2<H2>(a[i]);
      const uint32_t b2 = __hgt2_mask(k, as_h2<H2>(t3));
      const uint32_t b1 = __hgt2_mask(k, as_h2<H2>((t5 & b2) | (t1 & ~b2)));
      const uint32_t th = (t6 & b1) | (t4 & ~b1), tl = (t2 & b1) | (t0 & ~b1);
      const uint32_t b0 = __hgt2_mask(k, as_h2<H2>((th & b2) | (tl & ~b2)));
      const uint32_t code = (b2 & 0x00040004u) | (b1 & 0x00020002u) |
                            (b0 & 0x00010001u) |
                            ((p[i] >> 12) & 0x00080008u);  // the sign bits
      const uint32_t byte = (code & 0xFu) | ((code >> 12) & 0xF0u);
      if (i < 4)
        w0 |= byte << (8 * i);
      else
        w1 |= byte << (8 * (i - 4));
    }
  }
  return static_cast<uint8_t>(sb);
}

// Eight values x (fp32 bit patterns, x[0] first) -> four bytes of e2m1
// codes (element 2i in the low nibble of byte i) of q = x * rh + RN(x * rl),
// rounded once (packed fma), by the hardware conversion (round to nearest
// even, saturating at 6, sign kept).
__device__ __forceinline__ uint32_t e2m1_scaled8(const uint32_t (&x)[8],
                                                 float rh, float rl) {
  uint32_t r;
  asm("{\n\t"
      ".reg .b64 V, P, RH, RL;\n\t"
      ".reg .b32 q0, q1, q2, q3, q4, q5, q6, q7;\n\t"
      ".reg .b8 c0, c1, c2, c3;\n\t"
      "mov.b64 RH, {%9, %9};\n\t"
      "mov.b64 RL, {%10, %10};\n\t"
      "mov.b64 V, {%1, %2};\n\t"
      "mul.rn.f32x2 P, V, RL;\n\t"
      "fma.rn.f32x2 V, V, RH, P;\n\t"
      "mov.b64 {q0, q1}, V;\n\t"
      "mov.b64 V, {%3, %4};\n\t"
      "mul.rn.f32x2 P, V, RL;\n\t"
      "fma.rn.f32x2 V, V, RH, P;\n\t"
      "mov.b64 {q2, q3}, V;\n\t"
      "mov.b64 V, {%5, %6};\n\t"
      "mul.rn.f32x2 P, V, RL;\n\t"
      "fma.rn.f32x2 V, V, RH, P;\n\t"
      "mov.b64 {q4, q5}, V;\n\t"
      "mov.b64 V, {%7, %8};\n\t"
      "mul.rn.f32x2 P, V, RL;\n\t"
      "fma.rn.f32x2 V, V, RH, P;\n\t"
      "mov.b64 {q6, q7}, V;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c0, q1, q0;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c1, q3, q2;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c2, q5, q4;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 c3, q7, q6;\n\t"
      "mov.b32 %0, {c0, c1, c2, c3};\n\t"
      "}"
      : "=r"(r)
      : "r"(x[0]), "r"(x[1]), "r"(x[2]), "r"(x[3]), "r"(x[4]), "r"(x[5]),
        "r"(x[6]), "r"(x[7]), "f"(rh), "f"(rl));
  return r;
}

// One block's scale byte e4m3(amax / 6) and the e2m1 codes of its sixteen
// values x (fp32 bit patterns) under it, with v / s replaced by
// v * rh + RN(v * rl), rounded once, where rh = 1/s rounded toward zero and
// rl = RN((1 - s * rh) * rh) >= 0 (the residual 1 - s * rh is exact in one
// fma), and q rounded to e2m1 by the hardware conversion.  rh + rl is 1/s
// to about 2^-46 relative, so q is v / s to about 2^-45 relative:
//  * v / s exactly on a midpoint t (v = t * s) lands exactly on t and takes
//    the same tie rule;
//  * otherwise v / s lies at least ~2^-29 relative away from every fp32
//    rounding boundary t +- ulp(t) / 2 (v = (t +- ulp(t) / 2) * s would need
//    25 significant bits), so RN(q) and RN(v / s) fall on the same side of
//    t, or are both t.
// rl >= 0 keeps the sign of -0 (x * rl = -0); values whose quotient
// overflows saturate at 6 either way.  For 16-bit v, tests/test_oracle.py
// simulates this arithmetic for every finite value under every positive
// e4m3 s on the CPU, and a GPU test runs all of those pairs through the
// kernel; fp32 v are tested on and around every midpoint and boundary.
// (A single rounded reciprocal, q = RN(v * RN(1/s)), is not enough: ties
// at 1.25, 2.5 and 5 under scales of mantissa 1.875 round the wrong way.)
// (rh, rl) depend on the scale byte alone, so the kernel reads them from a
// 128-entry table in shared memory (rcp_pair fills it); a zero scale has
// (0, 0) and its codes are cleared by a select.
__device__ __forceinline__ float2 rcp_pair(uint32_t sb) {
  const float sd =
      __half2float(__half(__nv_cvt_fp8_to_halfraw(sb, __NV_E4M3)));
  if (!(sd > 0.f)) return make_float2(0.f, 0.f);
  const float rh = __frcp_rz(sd);
  return make_float2(rh, __fmul_rn(__fmaf_rn(-sd, rh, 1.0f), rh));
}
__device__ __forceinline__ uint8_t encode_rcp16(float amax,
                                                const uint32_t (&x)[16],
                                                uint32_t& w0, uint32_t& w1,
                                                const float2* rtab) {
  const __nv_fp8_storage_t sb =
      __nv_cvt_float_to_fp8(amax / 6.0f, __NV_SATFINITE, __NV_E4M3);
  const float2 r = rtab[sb & 0x7F];  // amax >= 0: the sign bit is clear
  const uint32_t(&xa)[8] = *reinterpret_cast<const uint32_t(*)[8]>(x);
  const uint32_t(&xb)[8] = *reinterpret_cast<const uint32_t(*)[8]>(x + 8);
  const uint32_t a = e2m1_scaled8(xa, r.x, r.y);
  const uint32_t b = e2m1_scaled8(xb, r.x, r.y);
  w0 = sb != 0 ? a : 0u;
  w1 = sb != 0 ? b : 0u;
  return static_cast<uint8_t>(sb);
}
// The same with (rh, rl) computed for the block: fp32 rows, for which the
// table lookup measured slower (25.8 against 25.2 us on 4096 x 7168).
__device__ __forceinline__ uint8_t encode_rcp16_direct(float amax,
                                                       const uint32_t (&x)[16],
                                                       uint32_t& w0,
                                                       uint32_t& w1) {
  const __nv_fp8_storage_t sb =
      __nv_cvt_float_to_fp8(amax / 6.0f, __NV_SATFINITE, __NV_E4M3);
  const float2 r = rcp_pair(sb);
  const uint32_t(&xa)[8] = *reinterpret_cast<const uint32_t(*)[8]>(x);
  const uint32_t(&xb)[8] = *reinterpret_cast<const uint32_t(*)[8]>(x + 8);
  w0 = 0;
  w1 = 0;
  if (sb != 0) {
    w0 = e2m1_scaled8(xa, r.x, r.y);
    w1 = e2m1_scaled8(xb, r.x, r.y);
  }
  return static_cast<uint8_t>(sb);
}

// The activation quantiser's 16-bit block form: amax as the largest |v| key
// (16-bit keys order like |v|), then encode_rcp16.  A block holding a NaN
// (key above +inf's) goes to the compare form.
template <typename H2>
__device__ __forceinline__ uint8_t quant_block16_x2(const uint32_t (&p)[8],
                                                    uint32_t& w0,
                                                    uint32_t& w1,
                                                    const float2* rtab) {
  using Ops = Half2Ops<H2>;
  uint32_t km = p[0] & 0x7FFF7FFFu;
#pragma unroll
  for (int i = 1; i < 8; ++i) km = __vmaxu2(km, p[i] & 0x7FFF7FFFu);
  const uint32_t key = max(km & 0xFFFFu, km >> 16);
  if (key > Ops::kInfKey) return quant_block16_x2_cmp<H2>(p, w0, w1);
  uint32_t x[16];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    x[2 * i] = __float_as_uint(Ops::lo(p[i]));
    x[2 * i + 1] = __float_as_uint(Ops::hi(p[i]));
  }
  return encode_rcp16(Ops::lo(key), x, w0, w1, rtab);
}

// The activation quantiser's fp32 block form: amax as the largest |v| bit
// pattern, then encode_rcp16_direct; a block holding a NaN goes to
// quant_block16.
__device__ __forceinline__ uint8_t quant_block16_rcp(const float (&v)[16],
                                                     uint32_t& w0,
                                                     uint32_t& w1) {
  uint32_t x[16];
  uint32_t km = 0;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    x[i] = __float_as_uint(v[i]);
    km = max(km, x[i] & 0x7FFFFFFFu);
  }
  if (km > 0x7F800000u) return quant_block16(v, w0, w1);
  return encode_rcp16_direct(__uint_as_float(km), x, w0, w1);
}

// Where the epilogue of one tile row writes its outputs: fp16 C, or NVFP4
// codes and blocked scales (KParams::cq).  `col0` is the tile's first column.
struct OutRow {
  __half* c;    // fp16: row `grow` of C at column col0
  uint8_t* q;   // NVFP4: the row's codes at column col0
  uint8_t* sf;  // NVFP4: the row's scale byte in atom 0 of its row block
  int col0;
  bool row_ok;  // grow < M: values / codes are stored
  bool sf_ok;   // grow < M rounded up to 128: scale bytes are stored (the
                // padding rows' scales are 0, their accumulators being 0)
};

// 32 outputs of one row -> 64 contiguous bytes of C.
// fp16(silu(x) * y) of 16 columns -> 32 bytes at dst (16-byte aligned).
__device__ __forceinline__ void store_row16(__half* dst, const float (&x)[16],
                                            const float (&y)[16]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint4 v;
    v.x = silu_mul_h2(x[8 * q + 0], x[8 * q + 1], y[8 * q + 0],
                      y[8 * q + 1]);
    v.y = silu_mul_h2(x[8 * q + 2], x[8 * q + 3], y[8 * q + 2],
                      y[8 * q + 3]);
    v.z = silu_mul_h2(x[8 * q + 4], x[8 * q + 5], y[8 * q + 4],
                      y[8 * q + 5]);
    v.w = silu_mul_h2(x[8 * q + 6], x[8 * q + 7], y[8 * q + 6],
                      y[8 * q + 7]);
    d[q] = v;
  }
}

__device__ __forceinline__ void store_row32(__half* dst, const float (&x)[32],
                                            const float (&y)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 v;
    v.x = silu_mul_h2(x[8 * q + 0], x[8 * q + 1], y[8 * q + 0],
                      y[8 * q + 1]);
    v.y = silu_mul_h2(x[8 * q + 2], x[8 * q + 3], y[8 * q + 2],
                      y[8 * q + 3]);
    v.z = silu_mul_h2(x[8 * q + 4], x[8 * q + 5], y[8 * q + 4],
                      y[8 * q + 5]);
    v.w = silu_mul_h2(x[8 * q + 6], x[8 * q + 7], y[8 * q + 6],
                      y[8 * q + 7]);
    d[q] = v;
  }
}

// Where a linear tile lies: its batch (or group) l, its tile coordinates in
// that problem, and the problem's rows (first row in A / SFA / C, count).
struct TileLoc {
  int l, m_tile, n_tile, row0, rows;
};

__device__ __forceinline__ TileLoc locate(const KParams& p, int tile) {
  TileLoc t;
  if (p.groups.count == 0) {
    tile_lmn(p.plan, tile, t.l, t.m_tile, t.n_tile);
    t.row0 = 0;
    t.rows = p.M;
    return t;
  }
  // the last group whose first tile is <= tile (empty groups have no tiles)
  int lo = 0, hi = p.groups.count - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.groups.tile0[mid] <= tile)
      lo = mid;
    else
      hi = mid - 1;
  }
  const int local = tile - p.groups.tile0[lo];
  const int span = kBM * p.plan.ctas;
  const int mt = (p.groups.rows[lo] + span - 1) / span;
  t.l = lo;
  t.n_tile = local / mt;
  t.m_tile = local - t.n_tile * mt;
  t.row0 = p.groups.row0[lo];
  t.rows = p.groups.rows[lo];
  return t;
}

// Output row `grow` (counted within the tile's problem) of the tile at `t`.
__device__ __forceinline__ OutRow out_row(const KParams& p, const TileLoc& t,
                                          int grow, int col0) {
  OutRow o;
  o.col0 = col0;
  o.row_ok = grow < t.rows;
  // rows of C before this one: whole earlier batches, or the group's offset
  const size_t r = (size_t)t.l * (p.groups.count ? 0 : p.M) + t.row0 + grow;
  if (p.cq != nullptr) {
    o.c = nullptr;
    o.q = p.cq + r * (p.N / 2) + col0 / 2;
    const int sr = t.row0 + grow;  // row in its blocked scale layout
    o.sf = p.sfc + (size_t)(p.groups.count ? 0 : t.l) * p.sfc_batch +
           (size_t)(sr / 128) * (p.N / 64) * kSfAtomBytes + (sr % 32) * 16 +
           ((sr % 128) / 32) * 4;
    o.sf_ok = grow < (t.rows + 127) / 128 * 128;
  } else {
    o.c = p.C + r * p.N + col0;
    o.q = nullptr;
    o.sf = nullptr;
    o.sf_ok = false;
  }
  return o;
}

// NVFP4 output of 16 consecutive columns of one row, given the fp16 values
// the fp16 output would hold (h, in pairs): quantised as one block, 8 bytes
// of codes at q and the e4m3 scale of column `col` of the row's blocked
// scales at sf.  Not inlined, and given its data by value: the epilogues,
// which serve the fp16 and the NVFP4 output, then carry one call instead of
// a copy of the quantiser at every output site (less code for the
// instruction cache) and keep their values in registers.
__device__ __noinline__ void quant_store16(uint8_t* q, uint8_t* sf, int col,
                                          bool row_ok, bool sf_ok,
                                          uint32_t h0, uint32_t h1,
                                          uint32_t h2, uint32_t h3,
                                          uint32_t h4, uint32_t h5,
                                          uint32_t h6, uint32_t h7) {
  const uint32_t h[8] = {h0, h1, h2, h3, h4, h5, h6, h7};
  uint32_t w0, w1;
  const uint8_t sb = quant_block16_x2_cmp<__half2>(h, w0, w1);
  if (row_ok) *reinterpret_cast<uint2*>(q) = make_uint2(w0, w1);
  if (sf_ok) sf[(col / 64) * kSfAtomBytes + (col / 16) % 4] = sb;
}

// NVFP4 output of tile columns [cc, cc + 16) of one row: fp16(silu(x) * y)
// quantised as one block.
__device__ __forceinline__ void quant_emit16(const OutRow& o, int cc,
                                             const float* x, const float* y) {
  uint32_t h[8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
    h[i] = silu_mul_h2(x[2 * i], x[2 * i + 1], y[2 * i], y[2 * i + 1]);
  quant_store16(o.q + cc / 2, o.sf, o.col0 + cc, o.row_ok, o.sf_ok, h[0],
                h[1], h[2], h[3], h[4], h[5], h[6], h[7]);
}

// Outputs of tile columns [cc, cc + 16) / [cc, cc + 32) of one row.
__device__ __forceinline__ void emit16(const OutRow& o, int cc,
                                       const float (&x)[16],
                                       const float (&y)[16]) {
  if (o.q == nullptr) {
    if (o.row_ok) store_row16(o.c + cc, x, y);
  } else {
    quant_emit16(o, cc, x, y);
  }
}

__device__ __forceinline__ void emit32(const OutRow& o, int cc,
                                       const float (&x)[32],
                                       const float (&y)[32]) {
  if (o.q == nullptr) {
    if (o.row_ok) store_row32(o.c + cc, x, y);
  } else {
    quant_emit16(o, cc, x, y);
    quant_emit16(o, cc + 16, x + 16, y + 16);
  }
}

// fp16(silu(x) * y) of 32 columns of one row into a C store box, whose
// rows are 128 bytes in the 128-byte-swizzled layout of the C tensor map:
// 16-byte chunk j of box row r sits at chunk j ^ (r % 8), so the 32 rows of
// a warp write all banks.  `j0` is the first chunk (4 per 32 columns).
__device__ __forceinline__ void stage_row32(uint8_t* row_base, int r, int j0,
                                            const float (&x)[32],
                                            const float (&y)[32]) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 v;
    v.x = silu_mul_h2(x[8 * q + 0], x[8 * q + 1], y[8 * q + 0],
                      y[8 * q + 1]);
    v.y = silu_mul_h2(x[8 * q + 2], x[8 * q + 3], y[8 * q + 2],
                      y[8 * q + 3]);
    v.z = silu_mul_h2(x[8 * q + 4], x[8 * q + 5], y[8 * q + 4],
                      y[8 * q + 5]);
    v.w = silu_mul_h2(x[8 * q + 6], x[8 * q + 7], y[8 * q + 6],
                      y[8 * q + 7]);
    sts128(smem_u32(row_base + (((j0 + q) ^ (r & 7)) << 4)), v);
  }
}

// The same for 16 columns: 16-byte chunks j0 and j0 + 1 of the box row.
__device__ __forceinline__ void stage_row16(uint8_t* row_base, int r, int j0,
                                            const float (&x)[16],
                                            const float (&y)[16]) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint4 v;
    v.x = silu_mul_h2(x[8 * q + 0], x[8 * q + 1], y[8 * q + 0], y[8 * q + 1]);
    v.y = silu_mul_h2(x[8 * q + 2], x[8 * q + 3], y[8 * q + 2], y[8 * q + 3]);
    v.z = silu_mul_h2(x[8 * q + 4], x[8 * q + 5], y[8 * q + 4], y[8 * q + 5]);
    v.w = silu_mul_h2(x[8 * q + 6], x[8 * q + 7], y[8 * q + 6], y[8 * q + 7]);
    sts128(smem_u32(row_base + (((j0 + q) ^ (r & 7)) << 4)), v);
  }
}

// Where a whole tile's fp16 outputs go when they are stored with TMA.
struct CStore {
  uint8_t* box;  // box 0 (columns [0, 64)); box 1 follows (BN = 128)
  bool store;    // this CTA's 128 rows start below the problem's rows
  int x, y, z;   // byte column, row and batch of box 0 in the C map
};

// Epilogue of a whole tile in the 2-SM pair kernel, run by the four
// epilogue warps (thread = row), in phases of 64 columns of both GEMMs: a
// phase's four TMEM loads (128 registers) are issued before one wait, and
// the accumulator is released (on the even CTA's acc_empty barrier, cluster
// address `acc_empty_c`) as soon as the last phase's loads have completed.
// A TMEM load round trip costs ~500 cycles, far more than the math of 16
// columns, so the epilogue's length is set by the number of load waits:
// two here (BN = 128), against eight with 16-column chunks; and the next
// tile's MMAs wait for one phase of math only.  With `cs` (fp16 C) a
// phase's outputs go into its C store box and thread 0 stores the box with
// TMA once the four warps have written it (after the box's previous store
// has read it): a warp then writes shared memory 512 bytes per instruction
// where its row stores to global memory touched 32 rows at 16 bytes each,
// and the store engine writes whole lines.  Otherwise each thread stores
// its row.
template <int BN, bool TMA, typename Release>
__device__ __forceinline__ void tile_epilogue(uint32_t t_row, const OutRow& out,
                                              int row, Release release,
                                              const CStore& cs,
                                              const CUtensorMap* tmC,
                                              int c_layers) {
  constexpr int kPhases = BN / 64;
  if (TMA) {
    if (threadIdx.x == 0) bulk_wait_group_read0();
    epi_bar();
  }
#pragma unroll 1
  for (int ph = 0; ph < kPhases; ++ph) {
    float x0[32], x1[32], y0[32], y1[32];
    __syncwarp();
    tc_ld_32cols(t_row + 64 * ph, x0);
    tc_ld_32cols(t_row + 64 * ph + 32, x1);
    tc_ld_32cols(t_row + BN + 64 * ph, y0);
    tc_ld_32cols(t_row + BN + 64 * ph + 32, y1);
    tc_wait_ld();
    tie32(x0);
    tie32(x1);
    tie32(y0);
    tie32(y1);
    if (ph == kPhases - 1) release();
    if (!TMA) {
      emit32(out, 64 * ph, x0, y0);
      emit32(out, 64 * ph + 32, x1, y1);
      continue;
    }
    uint8_t* box = cs.box + ph * kCBoxBytes;
    stage_row32(box + row * 128, row, 0, x0, y0);
    stage_row32(box + row * 128, row, 4, x1, y1);
    fence_proxy_async_smem();  // the generic writes, before the TMA read
    epi_bar();
    if (threadIdx.x == 0 && cs.store) {
      if (c_layers > 1)
        tma_store_3d(tmC, box, cs.x + 128 * ph, cs.y, cs.z);
      else
        tma_store_2d(tmC, box, cs.x + 128 * ph, cs.y);
      bulk_commit_group();
    }
  }
}

// Stream-K partials: within a slot, 16-byte group g (4 consecutive columns;
// GEMM1 columns are groups [0, BN/4), GEMM2 columns [BN/4, BN/2)) of row r
// sits at float offset (g * 128 + r) * 4, so each warp store or load covers
// 512 contiguous bytes.  This writes the 32 columns of groups [g0, g0 + 8)
// of one row.
__device__ __forceinline__ void store_f32x32_t(float* slot, int g0, int row,
                                               const float (&v)[32]) {
  float4* d = reinterpret_cast<float4*>(slot);
#pragma unroll
  for (int q = 0; q < 8; ++q)
    __stcg(d + (size_t)(g0 + q) * 128 + row,
           make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]));
}

// Warp roles (352 threads, one CTA per SM):
//   warps 0-3   epilogue (warp w reads TMEM lanes 32w..32w+31 = tile rows)
//   warp 4      tile producer: lanes 0-2 issue the A, B1 and B2 tiles (TMA)
//               of a K block as one instruction
//   warp 5      scale producer: lanes 0-2 issue the three scale runs (bulk
//               copies) as one instruction, onto their own barrier
//   warp 6      TMEM owner and MMA issuer (one elected thread)
//   warps 7-10  scale warps, one per TMEM sub-partition (warp % 4)
// Per K block the scale warps read the 512-byte scale atoms from shared
// memory and write them into a per-stage TMEM region with tcgen05.st, each
// warp filling its own 32 lanes with the layout the block-scaled MMA reads:
// lane 32q+i, column c of a 4-column group holds the 4 scales of row
// i + 32c for that 64-wide K step — the row of the 128x4 atom.  Writing the
// scales from four warps keeps the MMA thread's instruction stream down to
// the four MMAs of the K block: every tcgen05 instruction costs its issuing
// thread ~50-70 cycles, and the K-block period is set by such single-thread
// instruction chains.  It also lets the B-operand scales of a 64-row tile
// (half an atom) sit next to each other, so both GEMMs always run as one MMA
// with N = 2 * BN over the stacked B1|B2 tile.
constexpr int kEpiWarps = 4;
constexpr int kProdAWarp = 4;
constexpr int kProdBWarp = 5;
constexpr int kMmaWarp = 6;
constexpr int kSfWarp0 = 7;
constexpr int kSfWarps = 4;
static_assert(kThreads == 32 * (kSfWarp0 + kSfWarps), "thread count");

// Owner side of a stream-K tile (the 128 epilogue threads, thread = row):
// adds the partials of the other contributors to this CTA's accumulator and
// writes C.  Called on the CTA's last item after its accumulator is complete,
// so the pipeline's stage buffers (`stage`, >= kFixSlots * 32 KB) are idle:
// the partials are staged through them by bulk copies, kFixSlots items of
// 32 KB (one contributor's 32 columns of both GEMMs for the 128 rows) in
// flight, instead of being loaded row by row by the threads themselves.
// `slot_ptr(b)` is contributor b's partial slot; `arrive_empty()` releases
// the accumulator after its last TMEM load.  Partials are added in
// contributor order, so the result does not depend on timing.
constexpr int kFixSlots = 4;
static_assert(kFixSlots == 4, "init_barriers_by_lane gives 4 lanes to them");
constexpr uint32_t kFixItemBytes = 32768;

template <int BN, typename SlotPtr, typename ArriveEmpty>
__device__ __forceinline__ void sk_owner_fixup(
    uint8_t* stage, uint64_t* fix_bar, int b_first, int b_last,
    SlotPtr slot_ptr, ArriveEmpty arrive_empty, uint32_t t_row, int row,
    const OutRow& out, unsigned* err) {
  const int nb = b_last - b_first;
  const int n_items = (BN / 32) * nb;
  uint64_t pol = 0;
  int issued = 0;  // thread 0: items whose copies have been issued
  auto issue = [&](int i) {
    ++issued;
    const int c = i / nb;
    const float* src = slot_ptr(b_first + 1 + i % nb);
    uint8_t* dst = stage + (i % kFixSlots) * kFixItemBytes;
    uint64_t* bar = &fix_bar[i % kFixSlots];
    mbar_arrive_expect_tx(bar, kFixItemBytes);
    bulk_load(dst, src + (size_t)(8 * c) * 128 * 4, kFixItemBytes / 2, bar,
              pol);
    bulk_load(dst + kFixItemBytes / 2,
              src + (size_t)(BN / 4 + 8 * c) * 128 * 4, kFixItemBytes / 2,
              bar, pol);
  };
  if (threadIdx.x == 0) {
    NVFP4DG_STAMP(4, 40);
    // the partials were acquired through the counter (generic proxy); the
    // copies read them through the async proxy
    fence_proxy_async_global();
    pol = kPolicyEvictFirst;
    for (int i = 0; i < n_items && i < kFixSlots; ++i) issue(i);
  }
#pragma unroll 1
  for (int c = 0; c < BN / 32; ++c) {
    float x[32], y[32];
    __syncwarp();
    tc_ld_32cols(t_row + 32 * c, x);
    tc_ld_32cols(t_row + BN + 32 * c, y);
    tc_wait_ld();
    if (c == BN / 32 - 1) arrive_empty();
#pragma unroll 1
    for (int j = 0; j < nb; ++j) {
      const int i = c * nb + j;
      // after a timeout every later wait returns at once (err is set); the
      // threads still meet at each barrier below
      mbar_wait(&fix_bar[i % kFixSlots], (i / kFixSlots) & 1, err,
                kErrEpilogue);
      if (threadIdx.x == 0 && i < 16) NVFP4DG_STAMP(5, 41 + i);
      const float4* sx = reinterpret_cast<const float4*>(
                             stage + (i % kFixSlots) * kFixItemBytes) +
                         row;
      const float4* sy = sx + kFixItemBytes / 2 / 16;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 a = sx[q * 128];
        const float4 b = sy[q * 128];
        x[4 * q] += a.x;
        x[4 * q + 1] += a.y;
        x[4 * q + 2] += a.z;
        x[4 * q + 3] += a.w;
        y[4 * q] += b.x;
        y[4 * q + 1] += b.y;
        y[4 * q + 2] += b.z;
        y[4 * q + 3] += b.w;
      }
      epi_bar();  // every thread is done with the slot
      if (threadIdx.x == 0 && i + kFixSlots < n_items) {
        fence_proxy_async_smem();  // generic reads before the async refill
        issue(i + kFixSlots);
      }
    }
    emit32(out, 32 * c, x, y);
    if (threadIdx.x == 0) NVFP4DG_STAMP(4, 41 + c);
  }
  // After a timeout, copies may still be in flight: let them land (bounded)
  // before the CTA can exit.
  if (threadIdx.x == 0 && *reinterpret_cast<volatile unsigned*>(err) != 0u) {
    for (int i = issued > kFixSlots ? issued - kFixSlots : 0; i < issued; ++i)
      mbar_wait(&fix_bar[i % kFixSlots], (i / kFixSlots) & 1, err, kErrDrain,
                /*bail_on_err=*/false);
  }
}

// 256-thread barrier (id 3) of the split-K epilogue (epilogue warps 0-3 and
// scale warps 7-10) that also ANDs a predicate.
__device__ __forceinline__ bool split_group_all(bool pred) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 3, 256, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"(static_cast<uint32_t>(pred))
      : "memory");
  return out != 0;
}

// Epilogue of a cluster split-K tile, run once by the four epilogue warps
// (part 0) and the four scale warps (part 1; idle once the main loop is
// done): each warp owns TMEM lanes 32 (warp % 4) .. + 31.  Each of the two
// CTAs holds the partial sums of half of K; CTA h finishes output columns
// [h BN/2, (h+1) BN/2) in 16-column chunks j, part (j % 2) taking chunk j.
// For each of its chunks a warp sends the peer's GEMM1 and GEMM2 partials of
// chunk j into the peer's operand ring (idle once the peer's MMAs are done)
// with st.async counted on the peer's barrier recv_bar[j]; then it adds the
// peer's partials of its own chunks as they land, so the combine of early
// chunks overlaps the exchange of later ones.  In the exchange buffer the
// 16-byte group g of row r sits at (g * 128 + r) * 16 (GEMM1 chunk j: groups
// 4j .. 4j+3, GEMM2 chunk j: groups 4 (BN/32 + j) ..), so a warp's 32 rows
// are contiguous.
// `own` is the half of K this CTA computed, which is also the half of the
// columns it finishes; `xpeer` the cluster rank of the CTA that holds the
// other half of K for the same 128 output rows; `grow0` the first of those
// rows in C.  With `cluster_waited` set, the cluster barrier that publishes
// every CTA's barrier initialisation has already been waited on.
template <int BN>
__device__ __forceinline__ void split_epilogue(
    const KParams& p, uint8_t* smem, uint32_t tmem, uint64_t* acc_full_bar,
    uint64_t* ready_bar, uint64_t* recv_bar, int warp, int lane, int part,
    int own, uint32_t xpeer, const TileLoc& loc, int grow0, int n_tile,
    bool& cluster_waited, uint8_t* cbox = nullptr,
    const CUtensorMap* tmC = nullptr) {
  constexpr int kHalf = BN / 2;
  constexpr int kHalfChunks = kHalf / 16;
  constexpr uint32_t kChunkBytes = 2u * 128u * 16u * 4u;  // GEMM1 + GEMM2
  const int other = own ^ 1;
  const int row = 32 * (warp % 4) + lane;
  const uint32_t t_row = tmem + (static_cast<uint32_t>(32 * (warp % 4)) << 16);
  const int grow = grow0 + row;
  const OutRow out = out_row(p, loc, grow, n_tile * BN);

  griddep_wait();  // global memory only after the previous grid
  bool ok = mbar_wait(acc_full_bar, 0, p.err, kErrEpilogue);
  if (!split_group_all(ok)) return;
  if (part == 0 && threadIdx.x == 0) NVFP4DG_STAMP(4, 0);
  tc_fence_after();
  if (!cluster_waited) {
    cluster_wait();  // the peer's barriers are initialised
    cluster_waited = true;
  }
  if (part == 0 && threadIdx.x == 0) {
#pragma unroll
    for (int c = 0; c < kHalfChunks; ++c)
      mbar_arrive_expect_tx(&recv_bar[c], kChunkBytes);
    mbar_arrive_cluster(mapa_shared(smem_u32(ready_bar), xpeer));
  }
  // This warp's chunks j = part, part + 2 (at most two): every TMEM load —
  // the peer's columns (`v`, sent) and this CTA's own (`ox`, `oy`, kept) —
  // is issued before one wait, which overlaps the wait for the peer.
  constexpr int kMine = (kHalfChunks + 1) / 2;
  float v[kMine][2][16];
  float ox[kMine][16], oy[kMine][16];
#pragma unroll
  for (int i = 0; i < kMine; ++i) {
    const int c = part + 2 * i;
    if (c < kHalfChunks) {
#pragma unroll
      for (int xy = 0; xy < 2; ++xy)
        tc_ld_16cols(t_row + static_cast<uint32_t>(xy * BN + other * kHalf +
                                                   16 * c),
                     v[i][xy]);
      tc_ld_16cols(t_row + own * kHalf + 16 * c, ox[i]);
      tc_ld_16cols(t_row + BN + own * kHalf + 16 * c, oy[i]);
    }
  }
  tc_wait_ld();
  ok = mbar_wait(ready_bar, 0, p.err, kErrEpilogue);
  if (!split_group_all(ok)) return;
  if (part == 0 && threadIdx.x == 0) NVFP4DG_STAMP(8, 41);
  const uint32_t xbuf = smem_u32(smem);
  const uint32_t xdst = mapa_shared(xbuf, xpeer);
#pragma unroll
  for (int i = 0; i < kMine; ++i) {
    const int c = part + 2 * i;
    if (c < kHalfChunks) {
      const uint32_t cbar = mapa_shared(smem_u32(&recv_bar[c]), xpeer);
#pragma unroll
      for (int xy = 0; xy < 2; ++xy) {
        const int g0 = 4 * (xy * kHalfChunks + c);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float g[4] = {v[i][xy][4 * q], v[i][xy][4 * q + 1],
                              v[i][xy][4 * q + 2], v[i][xy][4 * q + 3]};
          st_async_v4(xdst + ((g0 + q) * 128u + row) * 16u, g, cbar);
        }
      }
    }
  }
  if (part == 0 && threadIdx.x == 0) NVFP4DG_STAMP(8, 42);
  bool all_ok = true;
  // Own chunks: each as soon as the peer's partials of it have landed.
  if (part == 0 && threadIdx.x == 0) NVFP4DG_STAMP(8, 43);
#pragma unroll
  for (int i = 0; i < kMine; ++i) {
    const int c = part + 2 * i;
    if (c >= kHalfChunks) continue;
    all_ok = mbar_wait(&recv_bar[c], 0, p.err, kErrEpilogue) && all_ok;
    if (part == 0 && threadIdx.x == 0) NVFP4DG_STAMP(8, 44 + i);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint4 rx = lds128(xbuf + ((c * 4 + q) * 128u + row) * 16u);
      const uint4 ry =
          lds128(xbuf + (((kHalfChunks + c) * 4 + q) * 128u + row) * 16u);
      ox[i][4 * q + 0] += __uint_as_float(rx.x);
      ox[i][4 * q + 1] += __uint_as_float(rx.y);
      ox[i][4 * q + 2] += __uint_as_float(rx.z);
      ox[i][4 * q + 3] += __uint_as_float(rx.w);
      oy[i][4 * q + 0] += __uint_as_float(ry.x);
      oy[i][4 * q + 1] += __uint_as_float(ry.y);
      oy[i][4 * q + 2] += __uint_as_float(ry.z);
      oy[i][4 * q + 3] += __uint_as_float(ry.w);
    }
    // after an expired wait the values are stale but every access stays in
    // bounds; the error word reports it
    if (kHalf == 64 && cbox != nullptr)
      stage_row16(cbox + row * 128, row, 2 * c, ox[i], oy[i]);
    else
      emit16(out, own * kHalf + 16 * c, ox[i], oy[i]);
  }
  if (kHalf == 64 && cbox != nullptr) fence_proxy_async_smem();
  split_group_all(all_ok);  // every participant finishes the tile together
  // With a C store box (fp16 C, 64 columns per half): the half-tile's 128
  // rows x 64 columns go out as one TMA store.
  if (kHalf == 64 && cbox != nullptr && threadIdx.x == 0 && grow0 < loc.rows) {
    const int bx = (n_tile * BN + own * kHalf) * 2;
    if (p.c_layers > 1)
      tma_store_3d(tmC, cbox, bx, grow0, loc.l);
    else
      tma_store_2d(tmC, cbox, bx, grow0);
    bulk_commit_group();
  }
  tc_fence_before();
  if (part == 0 && threadIdx.x == 0) NVFP4DG_STAMP(5, 0);
}

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    dual_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB1,
                     const __grid_constant__ CUtensorMap tmB2,
                     const __grid_constant__ CUtensorMap tmC,
                     const __grid_constant__ KParams p) {
  using Cf = Cfg<BN>;
  constexpr int S = Cf::kStages;
  constexpr uint32_t kBytesA = Cf::kABytes;
  constexpr uint32_t kBytesB = 2 * Cf::kBBytes;
  constexpr uint32_t kBytesSf = 3 * kSfRunBytes;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[S];    // operands + scales ready
  __shared__ __align__(8) uint64_t sfdata_bar[S];  // scale runs landed
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t acc_full_bar;
  __shared__ __align__(8) uint64_t acc_empty_bar;
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ __align__(8) uint64_t ready_bar;  // split-K: peer may write
  __shared__ __align__(8) uint64_t fix_bar[kFixSlots];  // stream-K owner
  // split-K: the peer's partials of chunk j of this CTA's half landed
  __shared__ __align__(8) uint64_t recv_bar[BN / 32];
  __shared__ uint32_t tmem_base_sh;

  // Operand tiles use the 128-byte swizzle, whose pattern repeats every
  // 1024 bytes: align the ring to 1024 in the shared window.
  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  NVFP4DG_STAMP_NS(61);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  const Plan& plan = p.plan;

  const bool producer = (warp == kProdAWarp || warp == kProdBWarp);
  // Warp 0 (an epilogue warp, idle until the first tile is computed)
  // initialises the mbarriers while the producers work out their first item.
  if (warp == 0) {
    // full: the scale warps, the first one's arrival carrying the tiles'
    // bytes; sfdata: one arming arrival; empty: the MMAs' tcgen05.commit
    init_barriers_by_lane<S, BN / 32>(
        lane, full_bar, kSfWarps, sfdata_bar, empty_bar, &acc_full_bar,
        &acc_empty_bar, 32 * kEpiWarps, &drain_bar, &ready_bar, fix_bar,
        recv_bar, kBytesSf);
    if (lane == 0) prefetch_tmap(&tmA);
    if (lane == 1) prefetch_tmap(&tmB1);
    if (lane == 2) prefetch_tmap(&tmB2);
  }
  // Split-K clusters: every thread arrives on the cluster barrier once the
  // barriers are initialised; the epilogue waits on it before its first
  // remote operation, the other warps at teardown.
  __syncwarp();
  if (plan.split == 2) cluster_arrive_relaxed();
  uint32_t tmem = 0;
  if (!producer) {
    if (warp == 0) named_bar_arrive(kBarInit, 96);
    if (warp == kMmaWarp) {
      tmem_alloc(&tmem_base_sh, kTmemCols);
      tmem_relinquish();
    }
    tc_fence_before();
    named_bar_sync(kBarStart, kThreads - 64);
    tc_fence_after();
    tmem = tmem_base_sh;
  }
  // Whether this thread has waited on that arrival (warp-uniform).
  bool cluster_waited = false;
  // Split-K: this CTA's half of K (= its cluster rank) and its tile.
  const int split_own = static_cast<int>(blockIdx.x & 1);
  const TileLoc split_loc = locate(p, static_cast<int>(blockIdx.x >> 1));
  const int split_m_tile = split_loc.m_tile, split_n_tile = split_loc.n_tile;
  // Everything above touched only this CTA's on-chip state; the inputs, C and
  // the workspace may be written by the previous grid in the stream.
  // Each role waits for the previous grid (griddepcontrol.wait) only after
  // its own setup, so the first pass through its code overlaps that wait.
  griddep_launch_dependents();
  NVFP4DG_STAMP_NS(62);
  const int kblk64 = p.K / 64;  // scale atoms per 128-row block

  if (warp == kProdAWarp || warp == kProdBWarp) {
    // ------------------------------------------------------------ producers
    // Lane 0 of warp 4 copies the A scale run and the A tile, lane 0 of
    // warp 5 the two B scale runs and the B tiles (one copy for B1 and B2
    // with the pair map).  A thread issues its copy instructions one at a
    // time (~100 cycles each, measured) while separate warps issue side by
    // side, so a K block's copies are split between two warps.  The
    // producers only copy; the expected bytes come from elsewhere: the first
    // scale warp's arrival on a stage's tile barrier carries the tiles'
    // bytes, and the same warp re-arms the stage's scale barrier for the
    // next fill once it has seen this one (the kernel's start arms the first
    // fills).  Keeping these off the MMA thread matters: its per-K-block
    // chain of waits and tcgen05 instructions sets the pace.  Scale runs go
    // first and land on their own barrier, so the scale warps move them into
    // TMEM while the tiles are in flight.
    // First item and its addresses before meeting warp 0 (parameters only).
    const bool a_side = (warp == kProdAWarp);
    if (a_side && lane == 0) NVFP4DG_STAMP(1, 56);
    // A is read by every CTA of its row of tiles: keep it in L2 longer
    const uint64_t pol = a_side ? kPolicyEvictLast : kPolicyEvictNormal;
    WorkIter it;
    work_begin(plan, blockIdx.x, it);
    if (a_side && lane == 0) NVFP4DG_STAMP(1, 57);
    Work w;
    bool have = work_next(plan, it, w);
    if (a_side && lane == 0) NVFP4DG_STAMP(1, 58);
    int l = 0, m_tile = 0, n_tile = 0;
    const uint8_t* sfa_src = nullptr;
    size_t sfb_off = 0;
    int a_row = 0, a_layer = 0;
    auto place = [&] {
      const TileLoc t = locate(p, w.tile);
      l = t.l;
      m_tile = t.m_tile;
      n_tile = t.n_tile;
      // A and SFA: rows of batch l, or the group's rows of the one matrix
      a_row = t.row0 + m_tile * kBM;
      a_layer = p.groups.count ? 0 : l;
      sfa_src = p.sfa + (size_t)a_layer * p.sfa_batch +
                (size_t)(a_row / kBM) * kblk64 * kSfAtomBytes;
      sfb_off = (size_t)l * p.sfb_batch +
                (size_t)((n_tile * BN) / 128) * kblk64 * kSfAtomBytes;
    };
    if (have) place();
    if (a_side && lane == 0) NVFP4DG_STAMP(1, 59);
    if (a_side && lane == 0) NVFP4DG_STAMP(1, 61);
    named_bar_sync(kBarInit, 96);  // the mbarriers are initialised
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      // global memory only after the previous grid, except for the weights
      // when the caller declares them unwritten by earlier kernels
      const bool w_early = p.static_weights != 0;
      if (a_side || !w_early) griddep_wait();
      if (a_side) NVFP4DG_STAMP(1, 62);
      while (ok && have) {
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (a_side) NVFP4DG_STAMP(9, issued);
          // a stage's first fill needs no wait: it is free from the start
          if (issued >= S &&
              !mbar_wait(&empty_bar[stage], phase ^ 1u, p.err, kErrProducer)) {
            ok = false;
            break;
          }
          if (a_side) NVFP4DG_STAMP(0, issued);
          uint8_t* st = smem + stage * Cf::kStageBytes;
          uint8_t* sf_dst = st + Cf::kABytes + 2 * Cf::kBBytes;
          const size_t run = (size_t)kb * kSfRunBytes;
          if (a_side) {
            bulk_load(sf_dst, sfa_src + run, kSfRunBytes, &sfdata_bar[stage],
                      pol);
            if (!w_early)
              bulk_load(sf_dst + kSfRunBytes, p.sfb1 + sfb_off + run,
                        kSfRunBytes, &sfdata_bar[stage], pol);
            tma_load_3d(st, &tmA, &full_bar[stage], kb * kRowBytes, a_row,
                        a_layer, pol);
          } else {
            if (w_early)
              bulk_load(sf_dst + kSfRunBytes, p.sfb1 + sfb_off + run,
                        kSfRunBytes, &sfdata_bar[stage], pol);
            bulk_load(sf_dst + 2 * kSfRunBytes, p.sfb2 + sfb_off + run,
                      kSfRunBytes, &sfdata_bar[stage], pol);
            // (the merged map's third coordinate picks B1 / B2; it is only
            // used for unbatched problems, otherwise it is the batch)
            tma_load_3d(st + Cf::kABytes, &tmB1, &full_bar[stage],
                        kb * kRowBytes, n_tile * BN, l, pol);
            if (!p.b_merged)
              tma_load_3d(st + Cf::kABytes + Cf::kBBytes, &tmB2,
                          &full_bar[stage], kb * kRowBytes, n_tile * BN, l,
                          pol);
          }
          if (a_side) NVFP4DG_STAMP(1, issued);
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        have = work_next(plan, it, w);
        if (have) place();
      }
      // Never leave with copies in flight: wait (bounded) until every stage
      // has completed the fill that holds this thread's last copies.
      for (int s = 0; s < S; ++s) {
        if (issued > s) {
          const uint32_t par =
              static_cast<uint32_t>(((issued - 1 - s) / S) & 1);
          mbar_wait(&sfdata_bar[s], par, p.err, kErrDrain,
                    /*bail_on_err=*/false);
          mbar_wait(&full_bar[s], par, p.err, kErrDrain,
                    /*bail_on_err=*/false);
        }
      }
    }
    __syncwarp();
  } else if (warp >= kSfWarp0) {
    // ------------------------------------------------------------ scale warps
    // This warp owns TMEM lanes 32q..32q+31; thread i writes lane 32q+i.
    const uint32_t q = static_cast<uint32_t>(warp % 4);
    const uint32_t t_lane = tmem + ((32u * q) << 16);
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    int done = 0;  // K blocks handed over (trace index)
    WorkIter it;
    work_begin(plan, blockIdx.x, it);
    Work w;
    bool have = work_next(plan, it, w);
    griddep_wait();  // global memory only after the previous grid
    for (; ok && have; have = work_next(plan, it, w)) {
      // BN = 64: the tile's B rows are one half of a 128-row atom, i.e.
      // atom words 2h and 2h+1 (rows 64h .. 64h+63).
      const int n_tile = locate(p, w.tile).n_tile;
      const int half = (BN == 64) ? (n_tile & 1) : 0;
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        const bool got = mbar_wait(&sfdata_bar[stage], phase, p.err, kErrMma);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        if (warp == kSfWarp0 && lane == 0) {
          NVFP4DG_STAMP(6, done);
          // arm the stage's next scale fill; it cannot complete before all
          // four scale warps have passed this fill (the copies wait for the
          // MMAs, which wait for every scale warp)
          mbar_arrive_expect_tx(&sfdata_bar[stage], kBytesSf);
        }
        const uint32_t sf_s = smem_u32(smem + stage * Cf::kStageBytes +
                                       Cf::kABytes + 2 * Cf::kBBytes) +
                              16u * lane;
        const uint32_t col = kSfTmemBase + stage * kSfTmemPerStage;
        uint32_t ra[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 v = lds128(sf_s + j * kSfAtomBytes);
          ra[4 * j + 0] = v.x;
          ra[4 * j + 1] = v.y;
          ra[4 * j + 2] = v.z;
          ra[4 * j + 3] = v.w;
        }
        __syncwarp();
        tc_st_16cols(t_lane + col, ra);
        if constexpr (BN == 128) {
          // per K step j: 4 columns of B1's atom, then 4 of B2's
          uint32_t rb[32];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 v1 = lds128(sf_s + kSfRunBytes + j * kSfAtomBytes);
            const uint4 v2 = lds128(sf_s + 2 * kSfRunBytes + j * kSfAtomBytes);
            rb[8 * j + 0] = v1.x;
            rb[8 * j + 1] = v1.y;
            rb[8 * j + 2] = v1.z;
            rb[8 * j + 3] = v1.w;
            rb[8 * j + 4] = v2.x;
            rb[8 * j + 5] = v2.y;
            rb[8 * j + 6] = v2.z;
            rb[8 * j + 7] = v2.w;
          }
          tc_st_32cols(t_lane + col + 16, rb);
        } else {
          // per K step j: B1 rows 0-31 / 32-63 of the tile, then B2's
          uint32_t rb[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 v1 = lds128(sf_s + kSfRunBytes + j * kSfAtomBytes);
            const uint4 v2 = lds128(sf_s + 2 * kSfRunBytes + j * kSfAtomBytes);
            rb[4 * j + 0] = half ? v1.z : v1.x;
            rb[4 * j + 1] = half ? v1.w : v1.y;
            rb[4 * j + 2] = half ? v2.z : v2.x;
            rb[4 * j + 3] = half ? v2.w : v2.y;
          }
          tc_st_16cols(t_lane + col + 16, rb);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          // the first scale warp's arrival also expects the tiles' bytes
          if (warp == kSfWarp0)
            mbar_arrive_expect_tx(&full_bar[stage], kBytesA + kBytesB);
          else
            mbar_arrive(&full_bar[stage]);
        }
        if (warp == kSfWarp0 && lane == 0) NVFP4DG_STAMP(7, done);
        ++done;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Split-K: the scale warps help finish the tile.
    if (plan.split == 2)
      split_epilogue<BN>(p, smem, tmem, &acc_full_bar, &ready_bar, recv_bar,
                         warp, lane, 1, split_own, split_own ^ 1u, split_loc,
                         split_m_tile * kBM, split_n_tile, cluster_waited);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_nvf4(128, 2 * BN);
      constexpr uint32_t kSfbStep = (BN == 128) ? 8u : 4u;
      const uint64_t a_desc0 = smem_desc(smem_u32(smem), 16, 1024,
                                         SmemLayout::kSwizzle128B);
      const uint64_t b_desc0 = smem_desc(smem_u32(smem) + Cf::kABytes, 16,
                                         1024, SmemLayout::kSwizzle128B);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      int consumed = 0;
      bool ok = true;
      WorkIter it;
      work_begin(plan, blockIdx.x, it);
      Work w;
      bool have = work_next(plan, it, w);
      griddep_wait();  // global memory only after the previous grid
      for (; ok && have; have = work_next(plan, it, w)) {
        if (!mbar_wait(&acc_empty_bar, acc_phase ^ 1u, p.err, kErrMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          // One wait per K block: the barrier completes when the tiles
          // have landed and all scale warps have written their scales.
          if (!mbar_wait(&full_bar[stage], phase, p.err, kErrMma)) {
            ok = false;
            break;
          }
          NVFP4DG_STAMP(2, consumed);
          tc_fence_after();  // orders the scale warps' tcgen05.st before us
          // Descriptors of stage `stage`, K step 0; a K step of 64 fp4 is
          // 32 bytes, i.e. +2 in the descriptors' address field (the field
          // holds address >> 4 and shared addresses stay below 2^18).
          const uint32_t soff = static_cast<uint32_t>(stage) *
                                (Cf::kStageBytes >> 4);
          const uint64_t a_desc = a_desc0 + soff;
          const uint64_t b_desc = b_desc0 + soff;
          const uint32_t sf_t = tmem + kSfTmemBase + stage * kSfTmemPerStage;
          const uint32_t acc0 = (kb > w.kb0) ? 1u : 0u;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            tc_mma_nvf4(tmem, a_desc + 2u * j, b_desc + 2u * j, kIdesc,
                        sf_t + 4 * j, sf_t + 16 + kSfbStep * j,
                        j > 0 ? 1u : acc0);
          }
          tc_commit(&empty_bar[stage]);
          NVFP4DG_STAMP(3, consumed);
          ++consumed;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full_bar);
        acc_phase ^= 1u;
      }
      // No MMA may still be running when TMEM is released.
      tc_commit(&drain_bar);
      mbar_wait(&drain_bar, 0, p.err, kErrDrain, /*bail_on_err=*/false);
    }
    __syncwarp();
  } else if (plan.split == 2) {
    // ------------------------------------------------------------ epilogue
    split_epilogue<BN>(p, smem, tmem, &acc_full_bar, &ready_bar, recv_bar,
                       warp, lane, 0, split_own, split_own ^ 1u, split_loc,
                       split_m_tile * kBM, split_n_tile, cluster_waited);
  } else {
    // ------------------------------------------------------------ epilogue
    const int row = threadIdx.x;  // TMEM lane == tile row
    const uint32_t t_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    uint32_t acc_phase = 0;
    int unit = 0;
    WorkIter it;
    work_begin(plan, blockIdx.x, it);
    Work w;
    bool have = work_next(plan, it, w);
    griddep_wait();  // global memory only after the previous grid
    for (; have; have = work_next(plan, it, w)) {
      const bool got = mbar_wait(&acc_full_bar, acc_phase, p.err, kErrEpilogue);
      if (!group_all<1>(got)) break;  // the four warps leave together
      if (threadIdx.x == 0) NVFP4DG_STAMP(4, unit);
      tc_fence_after();
      const TileLoc loc = locate(p, w.tile);
      const int n_tile = loc.n_tile;
      const int grow = loc.m_tile * kBM + row;
      const OutRow out = out_row(p, loc, grow, n_tile * BN);
      if (w.slot < 0) {
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          float x[32], y[32];
          __syncwarp();
          tc_ld_32cols(t_row + 32 * c, x);
          tc_ld_32cols(t_row + BN + 32 * c, y);
          tc_wait_ld();
          tie32(x);
          tie32(y);
          if (c == BN / 32 - 1) {
            tc_fence_before();
            mbar_arrive(&acc_empty_bar);
          }
          emit32(out, 32 * c, x, y);
        }
      } else {
        // A stream-K tile shared by CTAs b_first..b_last.  Its first K
        // blocks are b_first's last item, the later ones the others' first
        // items, so when b_first gets here the others have normally already
        // published their partials: it waits for their count, adds them to
        // its own accumulator and writes C; the others store a partial and
        // count it.
        const long long ts = w.tile - plan.dp_tiles;
        int b_first, b_last;
        sk_tile_owners(plan, ts, &b_first, &b_last);
        int* counter = p.counters + ts;
        if (static_cast<int>(blockIdx.x) != b_first) {
          float* mine =
              p.partials + (size_t)w.slot * partial_slot_floats(plan);
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            float x[32], y[32];
            __syncwarp();
            tc_ld_32cols(t_row + 32 * c, x);
            tc_ld_32cols(t_row + BN + 32 * c, y);
            tc_wait_ld();
            if (c == BN / 32 - 1) {
              tc_fence_before();
              mbar_arrive(&acc_empty_bar);
            }
            store_f32x32_t(mine, 8 * c, row, x);
            store_f32x32_t(mine, BN / 4 + 8 * c, row, y);
          }
          __threadfence();
          epi_bar();
          if (threadIdx.x == 0) red_release_add(counter, 1);
        } else {
          bool ready = true;
          if (threadIdx.x == 0) {
            NVFP4DG_STAMP(5, 40);
            ready = wait_count(counter, b_last - b_first + p.sk_extra, p.err,
                               kErrEpilogue, p.sk_wait_limit);
            if (ready) *counter = 0;  // ready for the next launch
          }
          if (!group_all<1>(ready)) break;
          sk_owner_fixup<BN>(
              smem, fix_bar, b_first, b_last,
              [&](int b) {
                return p.partials +
                       (size_t)sk_slot(plan, b, ts) * partial_slot_floats(plan);
              },
              [&] {
                tc_fence_before();
                mbar_arrive(&acc_empty_bar);
              },
              t_row, row, out, p.err);
        }
      }
      if (threadIdx.x == 0) NVFP4DG_STAMP(5, unit);
      ++unit;
      acc_phase ^= 1u;
    }
  }

  // ------------------------------------------------------------ teardown
  tc_fence_before();
  __syncthreads();
  // Split-K: neither CTA leaves while its peer may still write into it
  // (the epilogue warps have already waited on the start-up phase).
  if (plan.split == 2) {
    if (!cluster_waited) cluster_wait();
    cluster_sync_final();
  }
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
  NVFP4DG_STAMP_NS(63);
}

// ===========================================================================
// 2-SM pair kernel (cta_group::2): a cluster of two CTAs computes a
// 256 x BN tile of both GEMMs.  The even CTA issues M = 256, N = 2*BN MMAs;
// CTA r holds A rows [128r, 128r + 128) of the tile and the r-th half of the
// stacked B operand, i.e. the B1 tile in CTA 0 and the B2 tile in CTA 1, so
// each byte of B1 and B2 is loaded once per pair and every SM streams
// 16 + BN/8 KiB of operands per K block instead of 16 + BN/4 KiB.  Each CTA
// keeps its own scales in TMEM (its A rows, and all 2*BN B rows), and
// receives its 128 rows of the accumulator, so the epilogue is unchanged.
// Cross-CTA signals: both CTAs' A/B copies complete on the even CTA's
// `full` barrier; the odd CTA's scale warps and epilogue arrive remotely on
// the even CTA's `sf_ready` / `acc_empty`; the even CTA's MMA thread commits
// to both CTAs' `empty` / `acc_full` barriers.
// ===========================================================================
// Before the dependency wait of the 2-SM pair kernel, the epilogue warps
// (idle until the first accumulator is ready; lane 0 of warp q takes stages
// q, q + 4, ...) prefetch into L2 the operands of the first S stages of the
// CTA's first work item: its A rows and B half (tensor-map boxes) and the
// three scale runs.  A prefetch only warms L2, which is coherent, so it is
// correct whatever the previous grid writes; while the previous call drains,
// it turns the first stages' HBM latency into L2 latency.  Ungrouped
// problems with 2-D maps only.
template <int BN, int S>
__device__ __forceinline__ void pair_prefetch_first_stages(
    const KParams& p, const CUtensorMap* tmA, const CUtensorMap* tmB,
    int unit, int rank, int warp, int lane) {
  if (lane != 0 || p.maps3d || p.groups.count) return;
  WorkIter it;
  work_begin(p.plan, unit, it);
  Work w;
  if (!work_next(p.plan, it, w)) return;
  const TileLoc t = locate(p, w.tile);
  const int kblk64 = p.K / 64;
  const int a_row = t.m_tile * 2 * kBM + rank * kBM;
  const int a_blk = min(t.m_tile * 2 + rank, (t.rows + kBM - 1) / kBM - 1);
  const uint8_t* sfa = p.sfa + (size_t)a_blk * kblk64 * kSfAtomBytes;
  const size_t sfb_off = (size_t)((t.n_tile * BN) / 128) * kblk64 * kSfAtomBytes;
  const int nst = min(S, w.kb1 - w.kb0);
  for (int j = warp; j < nst; j += kEpiWarps) {
    const int kb = w.kb0 + j;
    const size_t run = (size_t)kb * kSfRunBytes;
    tma_prefetch_2d(tmA, kb * kRowBytes, a_row);
    tma_prefetch_2d(tmB, kb * kRowBytes, t.n_tile * BN);
    bulk_prefetch_l2(sfa + run, kSfRunBytes);
    bulk_prefetch_l2(p.sfb1 + sfb_off + run, kSfRunBytes);
    bulk_prefetch_l2(p.sfb2 + sfb_off + run, kSfRunBytes);
  }
}

template <int BN>
struct PairCfg {
  static constexpr int kStages = (BN == 128) ? 5 : 7;
  static constexpr int kABytes = kBM * kRowBytes;  // this CTA's A rows
  static constexpr int kBBytes = BN * kRowBytes;   // this CTA's B half
  static constexpr int kStageBytes = kABytes + kBBytes + 3 * kSfRunBytes;
  // BN = 128: this CTA's fp16 C tile (128 rows x 128 columns) staged for
  // the TMA store, two 16 KiB boxes of 64 columns, after the stages
  static constexpr int kCStageBytes = (BN == 128) ? 2 * kCBoxBytes : 0;
  static constexpr int kSmemBytes =
      kStages * kStageBytes + kCStageBytes + 1024;
  static constexpr int kSfBase = 2 * BN;  // scale regions follow the acc.
  static_assert(kStageBytes % 1024 == 0, "stages must stay 1024-B aligned");
  static_assert(kSmemBytes <= 227 * 1024, "shared memory budget");
  static_assert(kSfBase + kStages * kSfTmemPerStage <= kTmemCols,
                "TMEM budget");
  static_assert(kStages * kStageBytes >= 4 * 32768,
                "stream-K fixup staging reuses the stage buffers");
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1)
    dual_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ CUtensorMap tmB1,
                          const __grid_constant__ CUtensorMap tmB2,
                          const __grid_constant__ CUtensorMap tmC,
                          const __grid_constant__ KParams p) {
  using Cf = PairCfg<BN>;
  constexpr int S = Cf::kStages;

  extern __shared__ uint8_t smem_raw[];
  // even CTA: the A/B tiles of both CTAs landed and the scale warps of both
  // CTAs have written their scales
  __shared__ __align__(8) uint64_t full_bar[S];
  __shared__ __align__(8) uint64_t sfdata_bar[S];  // own scale runs landed
  __shared__ __align__(8) uint64_t empty_bar[S];
  __shared__ __align__(8) uint64_t acc_full_bar;
  __shared__ __align__(8) uint64_t acc_empty_bar;  // even CTA: both drained
  __shared__ __align__(8) uint64_t drain_bar;
  __shared__ __align__(8) uint64_t fix_bar[kFixSlots];  // stream-K owner
  __shared__ __align__(8) uint64_t ready_bar;  // split-K: partner may write
  // split-K: the partner's partials of chunk j of this CTA's half landed
  __shared__ __align__(8) uint64_t recv_bar[BN / 32];
  __shared__ uint32_t tmem_base_sh;

  const uint32_t raw_addr = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + (((raw_addr + 1023u) & ~1023u) - raw_addr);

  NVFP4DG_STAMP_NS(61);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x % 32;
  // Clusters of 2 CTAs (one pair), or of 4 for split-K (two pairs: ranks
  // 2h and 2h + 1 take half h of K).  A pair is ranks (lead, lead + 1).
  const uint32_t crank = cluster_ctarank();
  const uint32_t rank = crank & 1u;   // position in the pair
  const uint32_t lead = crank & ~1u;  // cluster rank of the pair's even CTA
  // Warp 0 initialises the mbarriers first of all: nothing of it depends on
  // the kernel parameters, whose first reads miss the constant cache (a new
  // parameter buffer each launch) and would otherwise delay every role
  // waiting for the barriers.
  if (warp == 0) {
    // full: the scale warps of both CTAs, on the even CTA the first one's
    // arrival carrying both CTAs' tile bytes; sfdata: one arming arrival;
    // empty: the MMA commit (even CTA) or the even producer A's forward
    init_barriers_by_lane<S, BN / 32>(
        lane, full_bar, 2 * kSfWarps, sfdata_bar, empty_bar, &acc_full_bar,
        &acc_empty_bar, 2 * kEpiWarps, &drain_bar, &ready_bar, fix_bar,
        recv_bar, 3 * kSfRunBytes);
    if (lane == 0) NVFP4DG_STAMP(9, 56);
    if (lane == 0) prefetch_tmap(&tmA);
    if (lane == 1) prefetch_tmap(rank == 0 ? &tmB1 : &tmB2);
  }
  // Every CTA's barriers initialised (published by the mbarrier-init fence)
  // before any remote use: arrive now, wait after the TMEM allocation, so
  // that the cluster-wide barrier completes meanwhile.
  __syncwarp();
  cluster_arrive_relaxed();
  const Plan& plan = p.plan;
  const int unit = blockIdx.x >> 1;   // the pair's work-unit index
  const bool leader = (rank == 0);
  // Split-K (4-CTA clusters): this pair's half of K, its tile, and the first
  // output row of this CTA's 128 rows; the partner is cluster rank crank ^ 2.
  const int split_own = static_cast<int>(crank >> 1);
  const TileLoc split_loc = locate(p, unit >> 1);
  const int split_m_tile = split_loc.m_tile, split_n_tile = split_loc.n_tile;
  const int split_grow0 =
      split_m_tile * 2 * kBM + static_cast<int>(rank) * kBM;
  bool cluster_waited = true;  // the start-up cluster barrier (below)
  const bool producer = (warp == kProdAWarp || warp == kProdBWarp);
  if (warp == 0 && lane == 2 && p.c_tma) prefetch_tmap(&tmC);
  uint32_t tmem = 0;
  if (!producer) {
    if (warp == 0) named_bar_arrive(kBarInit, 96);
    if (warp == kMmaWarp) {
      tmem_alloc_pair(&tmem_base_sh, kTmemCols);
      tmem_relinquish_pair();
      if (lane == 0) NVFP4DG_STAMP(9, 60);
    }
    tc_fence_before();
    named_bar_sync(kBarStart, kThreads - 64);  // TMEM base, barrier inits
    cluster_wait();
    tc_fence_after();
    tmem = tmem_base_sh;
  }
  // Each role waits for the previous grid (griddepcontrol.wait) only after
  // its own setup, so the first pass through its code overlaps that wait.
  griddep_launch_dependents();
  NVFP4DG_STAMP_NS(62);
  const int kblk64 = p.K / 64;

  if (warp == kProdAWarp || warp == kProdBWarp) {
    // ------------------------------------------------------------ producers
    // As in the 1-SM kernel, lane 0 of warp 4 copies this CTA's A scale run,
    // the first B scale run and its A rows, lane 0 of warp 5 the second B
    // scale run and this CTA's B half (the B1 tile in CTA 0, B2 in CTA 1):
    // a thread issues its copies one at a time, two warps side by side.
    // Tile bytes land on the even CTA's `full` barrier, whose expected bytes
    // (both CTAs' tiles) come with the even CTA's first scale warp's
    // arrival; scale runs land on this CTA's `sfdata` barrier, re-armed by
    // its first scale warp.
    // First item and its addresses before meeting warp 0 (parameters only).
    const bool a_side = (warp == kProdAWarp);
    // A is read by every CTA of its row of tiles: keep it in L2 longer
    const uint64_t pol = a_side ? kPolicyEvictLast : kPolicyEvictNormal;
    WorkIter it;
    work_begin(plan, unit, it);
    Work w;
    bool have = work_next(plan, it, w);
    int l = 0, n_tile = 0, a_row = 0, a_layer = 0;
    const uint8_t* sfa_src = nullptr;
    size_t sfb_off = 0;
    auto place = [&] {
      const TileLoc t = locate(p, w.tile);
      l = t.l;
      n_tile = t.n_tile;
      // A and SFA: rows of batch l, or the group's rows of the one matrix
      a_layer = p.groups.count ? 0 : l;
      a_row = t.row0 + t.m_tile * 2 * kBM + static_cast<int>(rank) * kBM;
      // A problem's SFA holds ceil(rows / 128) row blocks.  When the odd
      // CTA's 128 rows lie wholly past them (rows in (256t, 256t + 128] for
      // the last pair tile) it copies the last block instead: its A rows are
      // zero-filled by the tensor map (or belong to the next group) and its
      // accumulator rows are never stored.
      const int a_blk = t.row0 / kBM +
                        min(t.m_tile * 2 + static_cast<int>(rank),
                            (t.rows + kBM - 1) / kBM - 1);
      sfa_src = p.sfa + (size_t)a_layer * p.sfa_batch +
                (size_t)a_blk * kblk64 * kSfAtomBytes;
      sfb_off = (size_t)l * p.sfb_batch +
                (size_t)((n_tile * BN) / 128) * kblk64 * kSfAtomBytes;
    };
    if (have) place();
    named_bar_sync(kBarInit, 96);  // this CTA's mbarriers are initialised
    if (a_side && lane == 0) NVFP4DG_STAMP(9, 57);
    cluster_wait();                // and every other CTA's
    if (a_side && lane == 0) NVFP4DG_STAMP(9, 58);
    if (lane == 0) {
      const uint32_t full_c = mapa_shared(smem_u32(&full_bar[0]), lead);
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      // global memory only after the previous grid, except for the weights
      // when the caller declares them unwritten by earlier kernels
      const bool w_early = p.static_weights != 0;
      if (a_side || !w_early) griddep_wait();
      if (a_side) NVFP4DG_STAMP(9, 59);
      if (a_side) NVFP4DG_STAMP_NS_ANY(53);
      while (ok && have) {
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          if (issued >= S &&
              !mbar_wait_cluster(&empty_bar[stage], phase ^ 1u, p.err,
                                 kErrProducer)) {
            ok = false;
            break;
          }
          uint8_t* st = smem + stage * Cf::kStageBytes;
          uint8_t* sf_dst = st + Cf::kABytes + Cf::kBBytes;
          const size_t run = (size_t)kb * kSfRunBytes;
          const uint32_t full_s = full_c + 8u * static_cast<uint32_t>(stage);
          if (a_side) {
            NVFP4DG_STAMP(0, issued);
            // The MMAs that read this stage in both CTAs are done: pass that
            // on to the odd CTA (from the second fill on).
            if (leader && issued >= S)
              mbar_arrive_cluster(
                  mapa_shared(smem_u32(&empty_bar[stage]), lead + 1u));
            bulk_load(sf_dst, sfa_src + run, kSfRunBytes, &sfdata_bar[stage],
                      pol);
            if (!w_early)
              bulk_load(sf_dst + kSfRunBytes, p.sfb1 + sfb_off + run,
                        kSfRunBytes, &sfdata_bar[stage], pol);
            // unbatched problems use 2-D maps, batched ones 3-D maps whose
            // third coordinate is the batch
            if (!p.maps3d)
              tma_load_2d_pair(st, &tmA, full_s, kb * kRowBytes, a_row, pol);
            else
              tma_load_3d_pair(st, &tmA, full_s, kb * kRowBytes, a_row,
                               a_layer, pol);
            NVFP4DG_STAMP(1, issued);
          } else {
            if (w_early)
              bulk_load(sf_dst + kSfRunBytes, p.sfb1 + sfb_off + run,
                        kSfRunBytes, &sfdata_bar[stage], pol);
            bulk_load(sf_dst + 2 * kSfRunBytes, p.sfb2 + sfb_off + run,
                      kSfRunBytes, &sfdata_bar[stage], pol);
            if (!p.maps3d)
              tma_load_2d_pair(st + Cf::kABytes, rank == 0 ? &tmB1 : &tmB2,
                               full_s, kb * kRowBytes, n_tile * BN, pol);
            else
              tma_load_3d_pair(st + Cf::kABytes, rank == 0 ? &tmB1 : &tmB2,
                               full_s, kb * kRowBytes, n_tile * BN, l, pol);
          }
          ++issued;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        have = work_next(plan, it, w);
        if (have) place();
      }
      // Drain: the scale runs land on this CTA's own barrier; the A/B tiles
      // of both CTAs land on the even CTA's `full` barrier, which its warp 4
      // drains (the odd CTA cannot pass the final cluster barrier before
      // that).
      for (int s = 0; s < S; ++s) {
        if (issued > s) {
          const uint32_t par =
              static_cast<uint32_t>(((issued - 1 - s) / S) & 1);
          mbar_wait(&sfdata_bar[s], par, p.err, kErrDrain, false);
          if (a_side && leader)
            mbar_wait_cluster(&full_bar[s], par, p.err, kErrDrain, false);
        }
      }
    }
    __syncwarp();
  } else if (warp >= kSfWarp0) {
    // ------------------------------------------------------------ scale warps
    const uint32_t q = static_cast<uint32_t>(warp % 4);
    const uint32_t t_lane = tmem + ((32u * q) << 16);
    int stage = 0;
    uint32_t phase = 0;
    int done = 0;
    bool ok = true;
    WorkIter it;
    work_begin(plan, unit, it);
    Work w;
    bool have = work_next(plan, it, w);
    griddep_wait();  // global memory only after the previous grid
    for (; ok && have; have = work_next(plan, it, w)) {
      const int n_tile = locate(p, w.tile).n_tile;
      const int half = (BN == 64) ? (n_tile & 1) : 0;
      for (int kb = w.kb0; kb < w.kb1; ++kb) {
        const bool got =
            mbar_wait(&sfdata_bar[stage], phase, p.err, kErrMma);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        if (warp == kSfWarp0 && lane == 0) {
          NVFP4DG_STAMP(6, done);
          // arm the stage's next scale fill (see the 1-SM kernel)
          mbar_arrive_expect_tx(&sfdata_bar[stage], 3 * kSfRunBytes);
        }
        const uint32_t sf_s = smem_u32(smem + stage * Cf::kStageBytes +
                                       Cf::kABytes + Cf::kBBytes) +
                              16u * lane;
        const uint32_t col = Cf::kSfBase + stage * kSfTmemPerStage;
        uint32_t ra[16];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint4 v = lds128(sf_s + j * kSfAtomBytes);
          ra[4 * j + 0] = v.x;
          ra[4 * j + 1] = v.y;
          ra[4 * j + 2] = v.z;
          ra[4 * j + 3] = v.w;
        }
        __syncwarp();
        tc_st_16cols(t_lane + col, ra);
        if constexpr (BN == 128) {
          uint32_t rb[32];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 v1 = lds128(sf_s + kSfRunBytes + j * kSfAtomBytes);
            const uint4 v2 = lds128(sf_s + 2 * kSfRunBytes + j * kSfAtomBytes);
            rb[8 * j + 0] = v1.x;
            rb[8 * j + 1] = v1.y;
            rb[8 * j + 2] = v1.z;
            rb[8 * j + 3] = v1.w;
            rb[8 * j + 4] = v2.x;
            rb[8 * j + 5] = v2.y;
            rb[8 * j + 6] = v2.z;
            rb[8 * j + 7] = v2.w;
          }
          tc_st_32cols(t_lane + col + 16, rb);
        } else {
          uint32_t rb[16];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint4 v1 = lds128(sf_s + kSfRunBytes + j * kSfAtomBytes);
            const uint4 v2 = lds128(sf_s + 2 * kSfRunBytes + j * kSfAtomBytes);
            rb[4 * j + 0] = half ? v1.z : v1.x;
            rb[4 * j + 1] = half ? v1.w : v1.y;
            rb[4 * j + 2] = half ? v2.z : v2.x;
            rb[4 * j + 3] = half ? v2.w : v2.y;
          }
          tc_st_16cols(t_lane + col + 16, rb);
        }
        tc_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          const uint32_t full_s =
              mapa_shared(smem_u32(&full_bar[stage]), lead);
          // the even CTA's first scale warp also expects both CTAs' tiles
          if (leader && warp == kSfWarp0)
            mbar_arrive_expect_tx_cluster(full_s,
                                          2 * (Cf::kABytes + Cf::kBBytes));
          else
            mbar_arrive_cluster(full_s);
        }
        if (warp == kSfWarp0 && lane == 0) NVFP4DG_STAMP(7, done);
        ++done;
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // Split-K: the scale warps help finish the tile.
    if (plan.split == 2)
      split_epilogue<BN>(p, smem, tmem, &acc_full_bar, &ready_bar, recv_bar,
                         warp, lane, 1, split_own, crank ^ 2u, split_loc,
                         split_grow0, split_n_tile, cluster_waited,
                         p.c_tma ? smem + S * Cf::kStageBytes : nullptr, &tmC);
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0 && leader) {
      constexpr uint32_t kIdesc = idesc_nvf4(256, 2 * BN);
      constexpr uint32_t kSfbStep = (BN == 128) ? 8u : 4u;
      const uint32_t peer = lead + 1u;
      const uint64_t a_desc0 = smem_desc(smem_u32(smem), 16, 1024,
                                         SmemLayout::kSwizzle128B);
      const uint64_t b_desc0 = smem_desc(smem_u32(smem) + Cf::kABytes, 16,
                                         1024, SmemLayout::kSwizzle128B);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t acc_phase = 0;
      int consumed = 0;
      bool ok = true;
      WorkIter it;
      work_begin(plan, unit, it);
      Work w;
      bool have = work_next(plan, it, w);
      griddep_wait();  // global memory only after the previous grid
      for (; ok && have; have = work_next(plan, it, w)) {
        if (!mbar_wait_cluster(&acc_empty_bar, acc_phase ^ 1u, p.err,
                               kErrMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int kb = w.kb0; kb < w.kb1; ++kb) {
          // One wait per K block (tiles of both CTAs + all scales).
          if (!mbar_wait_cluster(&full_bar[stage], phase, p.err, kErrMma)) {
            ok = false;
            break;
          }
          NVFP4DG_STAMP(2, consumed);
          tc_fence_after();
          // Descriptors of stage `stage`, K step 0 (+2 per 32-byte K step).
          const uint32_t soff = static_cast<uint32_t>(stage) *
                                (Cf::kStageBytes >> 4);
          const uint64_t a_desc = a_desc0 + soff;
          const uint64_t b_desc = b_desc0 + soff;
          const uint32_t sf_t = tmem + Cf::kSfBase + stage * kSfTmemPerStage;
          const uint32_t acc0 = (kb > w.kb0) ? 1u : 0u;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            tc_mma_nvf4_pair(tmem, a_desc + 2u * j, b_desc + 2u * j, kIdesc,
                             sf_t + 4 * j, sf_t + 16 + kSfbStep * j,
                             j > 0 ? 1u : acc0);
          }
          // The stage is free in both CTAs once these MMAs complete; the
          // odd CTA learns it from the even producer A (one commit here).
          tc_commit_pair(mapa_shared(smem_u32(&empty_bar[stage]), lead));
          NVFP4DG_STAMP(3, consumed);
          ++consumed;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        const uint32_t ab = smem_u32(&acc_full_bar);
        tc_commit_pair(mapa_shared(ab, lead));
        tc_commit_pair(mapa_shared(ab, peer));
        acc_phase ^= 1u;
      }
      // The last unit's accumulator release (the odd CTA's epilogue warps
      // arrive here remotely) is awaited like the others, so that no arrival
      // is still in flight when the CTAs leave (cluster_sync_final).  Split-K
      // epilogues release nothing: their exchange is awaited by each side.
      if (ok && consumed > 0 && plan.split != 2)
        mbar_wait_cluster(&acc_empty_bar, acc_phase ^ 1u, p.err, kErrMma);
      tc_commit_pair(mapa_shared(smem_u32(&drain_bar), lead));
      mbar_wait(&drain_bar, 0, p.err, kErrDrain, /*bail_on_err=*/false);
    }
    __syncwarp();
  } else if (plan.split == 2) {
    // ------------------------------------------------------------ epilogue
    pair_prefetch_first_stages<BN, S>(p, &tmA, rank == 0 ? &tmB1 : &tmB2, unit,
                                      static_cast<int>(rank), warp, lane);
    split_epilogue<BN>(p, smem, tmem, &acc_full_bar, &ready_bar, recv_bar,
                       warp, lane, 0, split_own, crank ^ 2u, split_loc,
                       split_grow0, split_n_tile, cluster_waited,
                       p.c_tma ? smem + S * Cf::kStageBytes : nullptr, &tmC);
  } else {
    // ------------------------------------------------------------ epilogue
    pair_prefetch_first_stages<BN, S>(p, &tmA, rank == 0 ? &tmB1 : &tmB2, unit,
                                      static_cast<int>(rank), warp, lane);
    const int row = threadIdx.x;
    const uint32_t t_row = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const uint32_t acc_empty_c = mapa_shared(smem_u32(&acc_empty_bar), lead);
    // the accumulator may be overwritten: one arrival per warp on the even
    // CTA's barrier
    uint32_t acc_phase = 0;
    int unit_i = 0;
    auto release_acc = [&] {
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc_empty_c);
      if (threadIdx.x == 0) NVFP4DG_STAMP(8, unit_i);
    };
    WorkIter it;
    work_begin(plan, unit, it);
    Work w;
    bool have = work_next(plan, it, w);
    griddep_wait();  // global memory only after the previous grid
    for (; have; have = work_next(plan, it, w)) {
      const bool got =
          mbar_wait_cluster(&acc_full_bar, acc_phase, p.err, kErrEpilogue);
      if (!group_all<1>(got)) break;  // the four warps leave together
      if (threadIdx.x == 0) NVFP4DG_STAMP(4, unit_i);
      tc_fence_after();
      const TileLoc loc = locate(p, w.tile);
      const int n_tile = loc.n_tile;
      const int r0 = loc.m_tile * 2 * kBM + static_cast<int>(rank) * kBM;
      if (w.slot < 0 && p.c_tma) {
        // (only what this path needs is live across the epilogue: registers
        // are tight with a phase's 128 values)
        CStore cs;
        cs.box = smem + S * Cf::kStageBytes;
        cs.store = r0 < loc.rows;
        cs.x = n_tile * BN * 2;
        cs.y = r0;
        cs.z = loc.l;
        tile_epilogue<BN, true>(t_row, OutRow{}, row, release_acc, cs, &tmC,
                                p.c_layers);
      } else if (w.slot < 0) {
        const OutRow out = out_row(p, loc, r0 + row, n_tile * BN);
        tile_epilogue<BN, false>(t_row, out, row, release_acc, CStore{},
                                 &tmC, p.c_layers);
      } else {
        const OutRow out = out_row(p, loc, r0 + row, n_tile * BN);
        // Stream-K tile shared by units b_first..b_last: as in the 1-SM
        // kernel, unit b_first (for which these are its last K blocks) adds
        // the others' partials to its accumulator; each CTA of a pair deals
        // with its own 128 rows and its own counter.
        const long long ts = w.tile - plan.dp_tiles;
        int b_first, b_last;
        sk_tile_owners(plan, ts, &b_first, &b_last);
        int* counter = p.counters + ts * plan.ctas + rank;
        if (unit != b_first) {
          float* mine = p.partials +
                        (size_t)cta_slot(plan, w.slot, rank) *
                            partial_slot_floats(plan);
#pragma unroll 1
          for (int c = 0; c < BN / 32; ++c) {
            float x[32], y[32];
            __syncwarp();
            tc_ld_32cols(t_row + 32 * c, x);
            tc_ld_32cols(t_row + BN + 32 * c, y);
            tc_wait_ld();
            if (c == BN / 32 - 1) {
              tc_fence_before();
              __syncwarp();
              if (lane == 0) mbar_arrive_cluster(acc_empty_c);
            }
            store_f32x32_t(mine, 8 * c, row, x);
            store_f32x32_t(mine, BN / 4 + 8 * c, row, y);
          }
          __threadfence();
          epi_bar();
          if (threadIdx.x == 0) red_release_add(counter, 1);
        } else {
          bool ready = true;
          if (threadIdx.x == 0) {
            NVFP4DG_STAMP(5, 40);
            ready = wait_count(counter, b_last - b_first + p.sk_extra, p.err,
                               kErrEpilogue, p.sk_wait_limit);
            if (ready) *counter = 0;  // ready for the next launch
          }
          if (!group_all<1>(ready)) break;
          sk_owner_fixup<BN>(
              smem, fix_bar, b_first, b_last,
              [&](int b) {
                return p.partials +
                       (size_t)cta_slot(plan, sk_slot(plan, b, ts), rank) *
                           partial_slot_floats(plan);
              },
              [&] {
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_cluster(acc_empty_c);
              },
              t_row, row, out, p.err);
        }
      }
      if (threadIdx.x == 0) NVFP4DG_STAMP(5, unit_i);
      ++unit_i;
      acc_phase ^= 1u;
    }
  }

  // ------------------------------------------------------------ teardown
  // The C stores must have read their boxes before shared memory goes away;
  // their global writes complete before the grid does.
  if (lane == 0) NVFP4DG_STAMP(9, 40 + warp);
  NVFP4DG_STAMP_NS(50);
  if (p.c_tma && threadIdx.x == 0) bulk_wait_group_read0();
  NVFP4DG_STAMP_NS(51);
  tc_fence_before();
  cluster_sync_final();  // no CTA leaves while its peer may still signal it
  NVFP4DG_STAMP_NS(52);
  if (warp == kMmaWarp) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, kTmemCols);
  }
  NVFP4DG_STAMP_NS(63);
}

// ===========================================================================
// NVFP4 quantiser (fp32 rows -> e2m1 codes + e4m3 block scales)
// ===========================================================================
// Activation quantiser: rows of fp32 / fp16 / bf16 -> e2m1 codes and e4m3
// block scales, written straight into the blocked layout the dual GEMM
// reads.  One warp per 1024 consecutive elements of a row: lane i
// quantises the 16-element blocks at 16 i and 512 + 16 i, loading both
// (16-byte loads) before encoding either, so each warp load instruction
// covers one contiguous run of the row and its code stores 256 contiguous
// bytes; the four lanes of a 64-element group gather their scales into one
// 32-bit word for the plain layout and for the blocked one (row r's 16-byte
// atom row at (r % 32) * 16, quarter (r % 128) / 32 at +4 within it).  Warps
// of the padding rows up to a multiple of 128 write zero scales, so no
// memset of the blocked buffer is needed.  (One lane per row, each reading
// its own row, made every load instruction touch 32 cache lines: 54.4
// instead of 43.2 us on 8192 x 7168 bf16.)
template <typename T>
struct In16 {
  // 16 consecutive elements at p (16-byte aligned) as fp32
  static __device__ __forceinline__ void load(const T* p, float (&v)[16]);
};
template <>
struct In16<float> {
  static __device__ __forceinline__ void load(const float* p, float (&v)[16]) {
    const float4* s = reinterpret_cast<const float4*>(p);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 t = __ldg(s + q);
      v[4 * q] = t.x;
      v[4 * q + 1] = t.y;
      v[4 * q + 2] = t.z;
      v[4 * q + 3] = t.w;
    }
  }
};
// One 16-element block of a row: its raw loaded form and its encoder (fp32
// values through quant_block16_rcp; fp16 / bf16 kept as packed pairs for
// quant_block16_x2).
template <typename T>
struct Block16 {
  uint32_t raw[8];
  __device__ __forceinline__ void load(const T* p) {
    const uint4* s = reinterpret_cast<const uint4*>(p);
    const uint4 a = __ldg(s), b = __ldg(s + 1);
    raw[0] = a.x; raw[1] = a.y; raw[2] = a.z; raw[3] = a.w;
    raw[4] = b.x; raw[5] = b.y; raw[6] = b.z; raw[7] = b.w;
  }
  __device__ __forceinline__ uint8_t encode(uint32_t& w0, uint32_t& w1,
                                            const float2* rtab) const {
    using H2 = typename std::conditional<std::is_same<T, __half>::value,
                                         __half2, __nv_bfloat162>::type;
    return quant_block16_x2<H2>(raw, w0, w1, rtab);
  }
};
template <>
struct Block16<float> {
  float v[16];
  __device__ __forceinline__ void load(const float* p) { In16<float>::load(p, v); }
  __device__ __forceinline__ uint8_t encode(uint32_t& w0, uint32_t& w1,
                                            const float2*) const {
    return quant_block16_rcp(v, w0, w1);
  }
};

// One unit of the activation quantiser: the 1024-element run of row r that
// starts at element c0 - 16 lane (rows up to the next multiple of 128
// included: their scales are written as zero).
template <typename T>
__device__ __forceinline__ void quantize_unit(
    const T* __restrict__ X, int rows, int K, long long ldx,
    uint8_t* __restrict__ codes, uint8_t* __restrict__ sf_plain,
    uint8_t* __restrict__ sf_blocked, int groups, int lane, int r, int c0,
    const float2* rtab) {
  Block16<T> blk[2];
  bool act[2];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    act[h] = c0 + 512 * h < K;
    if (act[h] && r < rows) blk[h].load(X + (size_t)r * ldx + c0 + 512 * h);
  }
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int c = c0 + 512 * h;
    uint32_t sb = 0;
    if (act[h] && r < rows) {
      uint32_t w0, w1;
      sb = blk[h].encode(w0, w1, rtab);
      *reinterpret_cast<uint2*>(codes + (size_t)r * (K / 2) + c / 2) =
          make_uint2(w0, w1);
    }
    const uint32_t s1 = __shfl_down_sync(0xffffffffu, sb, 1);
    const uint32_t s2 = __shfl_down_sync(0xffffffffu, sb, 2);
    const uint32_t s3 = __shfl_down_sync(0xffffffffu, sb, 3);
    if ((lane & 3) == 0 && act[h]) {
      const uint32_t word = sb | (s1 << 8) | (s2 << 16) | (s3 << 24);
      const int g = c / 64;
      if (sf_plain != nullptr && r < rows)
        *reinterpret_cast<uint32_t*>(sf_plain + (size_t)r * (K / 16) +
                                     (size_t)g * 4) = word;
      *reinterpret_cast<uint32_t*>(
          sf_blocked + ((size_t)(r / 128) * groups + g) * kSfAtomBytes +
          (r % 32) * 16 + ((r % 128) / 32) * 4) = word;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
    quantize_rows_kernel(const T* __restrict__ X, int rows, int K, long long ldx,
                         uint8_t* __restrict__ codes,
                         uint8_t* __restrict__ sf_plain,
                         uint8_t* __restrict__ sf_blocked) {
  __shared__ float2 rtab[128];  // (rh, rl) of each e4m3 scale byte
  if (sizeof(T) == 2) {
    if (threadIdx.x < 128) rtab[threadIdx.x] = rcp_pair(threadIdx.x);
    __syncthreads();
  }
  const int groups = K / 64;
  const int chunks = (K + 1023) / 1024;  // 1024-element runs per row
  const int lane = threadIdx.x & 31;
  // unit u = row r, run ch (u = r * chunks + ch); each warp starts at its
  // global warp index and strides by the grid's warp count
  const long long u0 =
      (long long)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const long long stride = (long long)gridDim.x * (blockDim.x / 32);
  if (sizeof(T) == 2) {
    // 16-bit rows: (r, ch) advanced by (dr, dch) per step, one 64-bit
    // division per warp instead of one per unit (8192 x 7168 bf16, eager:
    // 31.4 instead of 33.1 us; the fp32 rows measured slower this way)
    const long long rows_pad = ((long long)rows + 127) / 128 * 128;
    long long r = u0 / chunks;
    int ch = static_cast<int>(u0 - r * chunks);
    const long long dr = stride / chunks;
    const int dch = static_cast<int>(stride - dr * chunks);
    for (; r < rows_pad; r += dr, ch += dch) {
      if (ch >= chunks) {
        ch -= chunks;
        if (++r >= rows_pad) break;
      }
      quantize_unit<T>(X, rows, K, ldx, codes, sf_plain, sf_blocked, groups,
                       lane, static_cast<int>(r), ch * 1024 + 16 * lane,
                       rtab);
    }
  } else {
    const long long units = ((long long)rows + 127) / 128 * 128 * chunks;
    for (long long u = u0; u < units; u += stride) {
      const int r = static_cast<int>(u / chunks);
      quantize_unit<T>(X, rows, K, ldx, codes, sf_plain, sf_blocked, groups,
                       lane, r,
                       static_cast<int>(u - (long long)r * chunks) * 1024 +
                           16 * lane,
                       rtab);
    }
  }
}

// Scale layout converter (plain [rows, K/16] <-> blocked).  One CTA moves
// a 128-row block x 32 four-scale groups (16 KiB) through shared memory:
// the plain side is read / written row by row (consecutive threads,
// consecutive 4-byte words of a row), the blocked side as whole 512-byte
// atoms (the 32 atoms of a row block and 32 consecutive groups are
// contiguous), so both sides are coalesced.  Padding rows of the blocked
// buffer are written as zero.  The shared tile is held in the blocked order,
// tile[group][word] with row r at word 4 (r % 32) + r / 32 and a row pitch
// of 129 words: the plain side (consecutive threads: consecutive groups of
// one row) and the blocked side (consecutive words of one atom) both touch
// 32 different banks per warp.  (With tile[row][group], rows r, r + 32,
// r + 64, r + 96 of one atom word run fell on one bank.)
constexpr int kCvtGroups = 32;
constexpr int kCvtPitch = 129;
__device__ __forceinline__ int cvt_word(int r) { return 4 * (r & 31) + (r >> 5); }
// words each of the 256 threads moves: a fixed count, so that every load of a
// thread is issued before the first one is used
constexpr int kCvtIters = 128 * kCvtGroups / 256;

__global__ void __launch_bounds__(256)
    scales_to_blocked_kernel(const uint8_t* __restrict__ plain, int rows,
                             int groups, long long ld,
                             uint8_t* __restrict__ blocked) {
  __shared__ uint32_t tile[kCvtGroups * kCvtPitch];
  const int rb = blockIdx.y;
  const int g0 = blockIdx.x * kCvtGroups;
  const int ng = min(kCvtGroups, groups - g0);
  uint32_t v[kCvtIters];
#pragma unroll
  for (int j = 0; j < kCvtIters; ++j) {
    const int i = threadIdx.x + j * 256;
    const int r = i / ng, gg = i - r * ng;
    const int row = rb * 128 + r;
    v[j] = (i < 128 * ng && row < rows)
               ? __ldg(reinterpret_cast<const uint32_t*>(
                     plain + (size_t)row * ld + 4 * (g0 + gg)))
               : 0u;
  }
#pragma unroll
  for (int j = 0; j < kCvtIters; ++j) {
    const int i = threadIdx.x + j * 256;
    const int r = i / ng, gg = i - r * ng;
    if (i < 128 * ng) tile[gg * kCvtPitch + cvt_word(r)] = v[j];
  }
  __syncthreads();
  uint32_t* out = reinterpret_cast<uint32_t*>(blocked) +
                  ((size_t)rb * groups + g0) * (kSfAtomBytes / 4);
  for (int i = threadIdx.x; i < 128 * ng; i += blockDim.x)
    out[i] = tile[(i >> 7) * kCvtPitch + (i & 127)];  // word i % 128 of atom i / 128
}

__global__ void __launch_bounds__(256)
    scales_from_blocked_kernel(const uint8_t* __restrict__ blocked, int rows,
                               int groups, long long ld,
                               uint8_t* __restrict__ plain) {
  __shared__ uint32_t tile[kCvtGroups * kCvtPitch];
  const int rb = blockIdx.y;
  const int g0 = blockIdx.x * kCvtGroups;
  const int ng = min(kCvtGroups, groups - g0);
  const uint32_t* in = reinterpret_cast<const uint32_t*>(blocked) +
                       ((size_t)rb * groups + g0) * (kSfAtomBytes / 4);
  uint32_t v[kCvtIters];
#pragma unroll
  for (int j = 0; j < kCvtIters; ++j) {
    const int i = threadIdx.x + j * 256;
    v[j] = i < 128 * ng ? __ldg(in + i) : 0u;
  }
#pragma unroll
  for (int j = 0; j < kCvtIters; ++j) {
    const int i = threadIdx.x + j * 256;
    if (i < 128 * ng) tile[(i >> 7) * kCvtPitch + (i & 127)] = v[j];
  }
  __syncthreads();
  for (int i = threadIdx.x; i < 128 * ng; i += blockDim.x) {
    const int r = i / ng, gg = i - r * ng;
    const int row = rb * 128 + r;
    if (row < rows)
      *reinterpret_cast<uint32_t*>(plain + (size_t)row * ld + 4 * (g0 + gg)) =
          tile[gg * kCvtPitch + cvt_word(r)];
  }
}

}  // namespace nvfp4dg

// ===========================================================================
// Host side
// ===========================================================================
namespace {

using namespace nvfp4dg;

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(NVFP4DG_ERR_CUDA,
              std::string(what) + ": " + cudaGetErrorString(e));
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                   void*, const cuuint64_t*, const cuuint64_t*,
                                   const cuuint32_t*, const cuuint32_t*,
                                   CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion,
                                   CUtensorMapFloatOOBfill);

std::mutex g_mu;
EncodeTiledFn g_encode = nullptr;

struct DevInfo {
  bool init = false;
  int sms = 0;
  int major = 0;
  int minor = 0;
  bool attr64 = false;
  bool attr128 = false;
  bool attr64p = false;
  bool attr128p = false;
  unsigned* err = nullptr;
};
std::map<int, DevInfo> g_dev;

// Bytes of a blocked scale tensor of `rows` rows and K / 16 scales a row.
long long blocked_scale_bytes(long long rows, long long K) {
  return (rows + 127) / 128 * (K / 64) * 512;
}

struct MapKey {
  const void* ptr;
  const void* ptr2;  // second tensor of a B1|B2 map, else nullptr
  int rank;
  long long rows;
  long long row_bytes;
  int box_rows;
  int dev;
  int layers;  // batch count (third dimension of a per-matrix map)
  bool operator<(const MapKey& o) const {
    if (ptr != o.ptr) return ptr < o.ptr;
    if (ptr2 != o.ptr2) return ptr2 < o.ptr2;
    if (rank != o.rank) return rank < o.rank;
    if (rows != o.rows) return rows < o.rows;
    if (row_bytes != o.row_bytes) return row_bytes < o.row_bytes;
    if (box_rows != o.box_rows) return box_rows < o.box_rows;
    if (layers != o.layers) return layers < o.layers;
    return dev < o.dev;
  }
};
std::map<MapKey, CUtensorMap> g_maps;

struct WsEntry {
  void* ptr = nullptr;
  size_t bytes = 0;
};
std::map<std::pair<int, void*>, WsEntry> g_ws;

int get_encode() {
  if (g_encode) return NVFP4DG_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn,
                                          cudaEnableDefault, &q);
  if (e != cudaSuccess || fn == nullptr || q != cudaDriverEntryPointSuccess)
    return fail(NVFP4DG_ERR_CUDA, "cuTensorMapEncodeTiled not available");
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return NVFP4DG_OK;
}

int device_info(int dev, DevInfo** out) {
  DevInfo& d = g_dev[dev];
  if (!d.init) {
    cudaError_t e;
    if ((e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount,
                                    dev)) != cudaSuccess)
      return cuda_fail(e, "cudaDeviceGetAttribute");
    cudaDeviceGetAttribute(&d.major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&d.minor, cudaDevAttrComputeCapabilityMinor, dev);
    if (d.major != 10)
      return fail(NVFP4DG_ERR_UNSUPPORTED,
                  "device is not sm_100 (compute capability " +
                      std::to_string(d.major) + "." + std::to_string(d.minor) +
                      ")");
    void* ptr = nullptr;
    if ((e = cudaGetSymbolAddress(&ptr, g_err_word)) != cudaSuccess)
      return cuda_fail(e, "cudaGetSymbolAddress(error word)");
    d.err = static_cast<unsigned*>(ptr);
    d.init = true;
  }
  *out = &d;
  return NVFP4DG_OK;
}

// Tiled map of a K-major [rows][row_bytes] matrix, box {128 B, box_rows}
// with the 128-byte swizzle.  rank 3 adds a unit outer dimension, so that
// the 1-SM kernel issues every tile copy as the same 3-D instruction (see
// b_pair_map).
// `layers` > 1: a batch of `layers` matrices of `rows` rows, one after the
// other (the third dimension, stride rows * row_bytes; needs rank 3).
int tensor_map(const void* ptr, long long rows, long long row_bytes,
               int box_rows, int dev, CUtensorMap* out, int rank = 2,
               int layers = 1) {
  MapKey key{ptr, nullptr, rank, rows, row_bytes, box_rows, dev, layers};
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return NVFP4DG_OK;
  }
  int rc = get_encode();
  if (rc) return rc;
  CUtensorMap m;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(row_bytes),
                              static_cast<cuuint64_t>(rows),
                              static_cast<cuuint64_t>(layers)};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_bytes),
                                 static_cast<cuuint64_t>(rows * row_bytes)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kRowBytes),
                             static_cast<cuuint32_t>(box_rows), 1};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, rank,
                        const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(NVFP4DG_ERR_CUDA,
                "cuTensorMapEncodeTiled failed (" + std::to_string((int)r) +
                    ")");
  if (g_maps.size() > 256) g_maps.clear();
  g_maps[key] = m;
  *out = m;
  return NVFP4DG_OK;
}

// One map over both weight matrices: a 3-D view [2][rows][row_bytes] whose
// outer stride is the distance from B1 to B2, so that a single copy with box
// {128 B, box_rows, 2} lands the B1 tile and then the B2 tile, exactly the
// stacked layout the MMA reads.  Every coordinate stays inside B1 or B2.
// Needs B2 above B1 at a multiple of 16 bytes; returns false (and the caller
// keeps one map per matrix) otherwise or if the driver rejects the view.
bool b_pair_map(const void* b1, const void* b2, long long rows,
                long long row_bytes, int box_rows, int dev, CUtensorMap* out) {
  const uintptr_t p1 = reinterpret_cast<uintptr_t>(b1);
  const uintptr_t p2 = reinterpret_cast<uintptr_t>(b2);
  if (p2 <= p1 || (p2 - p1) % 16 != 0 || (p2 - p1) >= (1ull << 40) ||
      static_cast<long long>(p2 - p1) < rows * row_bytes)
    return false;
  MapKey key{b1, b2, 3, rows, row_bytes, box_rows, dev, 1};
  auto it = g_maps.find(key);
  if (it != g_maps.end()) {
    *out = it->second;
    return true;
  }
  if (get_encode()) return false;
  CUtensorMap m;
  const cuuint64_t dims[3] = {static_cast<cuuint64_t>(row_bytes),
                              static_cast<cuuint64_t>(rows), 2};
  const cuuint64_t strides[2] = {static_cast<cuuint64_t>(row_bytes),
                                 static_cast<cuuint64_t>(p2 - p1)};
  const cuuint32_t box[3] = {static_cast<cuuint32_t>(kRowBytes),
                             static_cast<cuuint32_t>(box_rows), 2};
  const cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3,
                        const_cast<void*>(b1), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (g_maps.size() > 256) g_maps.clear();
  g_maps[key] = m;
  *out = m;
  return true;
}

// ---------------------------------------------------------------- planning
// Cost model (cycles of the busiest SM) used to pick the tile width, single
// CTA or 2-SM pair tiles, and whether to split tiles along K.  Measured on
// B200: an SM streams its operands from L2 at ~55 B/cycle whatever the copy
// sizes, so a K block costs max(bytes / 55, MMA cycles); the FP4 tensor pipe
// retires an M=128, N=256, K=64 MMA in ~128 cycles (N=128: ~70); the
// epilogue of a tile takes ~34 cycles per output column (not overlapped);
// a split tile costs its fp32 partial round trip through L2.
Plan plan_for(int M, int N, int K, int bn, int ctas, int unit_cap,
              bool streamk, bool force_sk, int L = 1) {
  Plan p{};
  p.bn = bn;
  p.ctas = ctas;
  p.L = L;
  p.m_tiles = (M + kBM * ctas - 1) / (kBM * ctas);
  p.n_tiles = N / bn;
  p.kblocks = K / 256;
  p.num_tiles = L * p.m_tiles * p.n_tiles;
  const int T = p.num_tiles;
  if (!streamk || (T % unit_cap == 0 && !force_sk)) {
    p.grid = std::min(T, unit_cap);
    p.dp_tiles = T;
    p.sk_iters = 0;
    set_tile_div(p);
    return p;
  }
  const int waves = T / unit_cap;
  p.dp_tiles = waves >= 2 ? (waves - 1) * unit_cap : 0;
  const long long sk_total = (long long)(T - p.dp_tiles) * p.kblocks;
  p.grid = (int)std::min<long long>(unit_cap, sk_total);
  if (p.dp_tiles > 0 && p.grid < unit_cap) p.grid = unit_cap;
  p.sk_iters = sk_total;
  set_tile_div(p);
  return p;
}

// Cluster split-K: each tile's K range in two halves on two work units (two
// CTAs, or two 2-SM pairs in a cluster of four) that exchange partial sums.
Plan plan_split(int M, int N, int K, int bn, int ctas = 1, int L = 1) {
  Plan p{};
  p.bn = bn;
  p.ctas = ctas;
  p.L = L;
  p.m_tiles = (M + kBM * ctas - 1) / (kBM * ctas);
  p.n_tiles = N / bn;
  p.kblocks = K / 256;
  p.num_tiles = L * p.m_tiles * p.n_tiles;
  p.grid = 2 * p.num_tiles;
  p.dp_tiles = p.num_tiles;
  p.sk_iters = 0;
  p.split = 2;
  set_tile_div(p);
  return p;
}

bool split_fits(int M, int N, int K, int bn, int sms, int ctas = 1,
                int L = 1) {
  if (N % bn != 0 || K / 256 < 2) return false;
  const long long tiles =
      (long long)L * ((M + kBM * ctas - 1) / (kBM * ctas)) * (N / bn);
  return 2 * ctas * tiles <= sms;
}

// Estimated SM cycles of the busiest work unit, from pipeline traces on B200
// (nvfp4_dual_gemm_b200.trace): the K-block period is set by the
// issuing threads' instruction chains (~700 cycles for N = 128 MMAs, ~710
// for 2-SM N = 256, ~790 for single-CTA N = 256); the first stage lands
// ~2300 cycles after start; an epilogue costs ~2100 / ~3900 cycles for
// BN = 64 / 128 (overlapped with the next tile's main loop except for a
// CTA's last tile); teardown ~500 cycles, ~2100 for 2-SM pairs.  Cluster
// split-K: a later first stage (~3200), ~830-cycle blocks (BN = 128), a
// ~5100-cycle exchange-and-combine epilogue (BN = 128; about half for 64)
// and ~1600 cycles of teardown.  Stream-K pays for its owners' partial
// fixups (below).
double plan_cost(const Plan& p) {
  const bool pair = (p.ctas == 2);
  const double per_block = pair ? (p.bn == 128 ? 710.0 : 700.0)
                                : (p.bn == 128 ? 790.0 : 715.0);
  const double epi = (p.bn == 128) ? 3900.0 : 2100.0;
  const double tear = pair ? 2100.0 : 500.0;
  const double start = 2300.0;
  if (p.split == 2) {
    // 2-SM pairs stream 38 KB per K block and SM where single CTAs stream
    // 54 KB (BN = 128) for the same MMAs; with ~128 SMs sharing L2 that
    // sets the block period
    const double blk = pair ? (p.bn == 128 ? 640.0 : 600.0)
                            : (p.bn == 128 ? 830.0 : 715.0);
    return (pair ? 3400.0 : 3200.0) + ((p.kblocks + 1) / 2) * blk +
           (p.bn == 128 ? 5100.0 : 2800.0) + (pair ? 2100.0 : 1600.0);
  }
  double cost = start + tear;
  double tiles = 0;
  if (p.dp_tiles > 0) {
    tiles = (double)((p.dp_tiles + p.grid - 1) / p.grid);
    cost += tiles * p.kblocks * per_block;
  }
  if (p.sk_iters > 0) {
    const double per_unit = (double)((p.sk_iters + p.grid - 1) / p.grid);
    const bool split = (p.sk_iters % p.grid) != 0 ||
                       ((p.sk_iters / p.grid) % p.kblocks) != 0;
    cost += per_unit * per_block;
    tiles += 2;
    if (split) {
      // The tile's owner stages the other contributors' partials through
      // shared memory, 32 KB per (contributor, 32-column chunk): ~3600
      // cycles to the first, then ~1250 (1-SM) / ~1800 (pair) per item
      // with every SM doing the same (measured); ~1500 more for the last
      // contributor's partial store.
      const double others =
          std::ceil((p.kblocks - 1) / per_unit);  // contributors - 1
      const double items = others * (p.bn / 32);
      cost += 1500.0 + 3600.0 + (items - 1.0) * (pair ? 1800.0 : 1250.0);
    }
  }
  // one exposed epilogue, the others mostly hidden behind the next tile
  cost += epi + (tiles > 1 ? (tiles - 1) * 0.3 * epi : 0.0);
  return cost;
}

// `L` independent problems of one shape (a batch) share one launch: their
// tiles are numbered batch by batch and scheduled together.
Plan choose_plan(int M, int N, int K, unsigned flags, int sms, int L = 1) {
  const int forced = static_cast<int>(flags & NVFP4DG_FLAG_GRID_MASK);
  const bool streamk = (flags & NVFP4DG_FLAG_NO_STREAMK) == 0;
  const bool force_sk = (flags & NVFP4DG_FLAG_FORCE_STREAMK) != 0;
  int bns[2];
  int nb = 0;
  if (flags & NVFP4DG_FLAG_BN64) {
    bns[nb++] = 64;
  } else if (flags & NVFP4DG_FLAG_BN128) {
    bns[nb++] = 128;
  } else {
    if (N % 128 == 0) bns[nb++] = 128;
    bns[nb++] = 64;
  }
  int ctas_opts[2];
  int nc = 0;
  if (!(flags & NVFP4DG_FLAG_NO_PAIR) && sms >= 2) ctas_opts[nc++] = 2;
  if (!(flags & NVFP4DG_FLAG_PAIR) || sms < 2) ctas_opts[nc++] = 1;
  Plan best{};
  double best_cost = 1e300;
  if (flags & NVFP4DG_FLAG_SPLITK) {
    // forced: 2-SM pairs when PAIR is also given, else single CTAs
    const int ctas = (flags & NVFP4DG_FLAG_PAIR) ? 2 : 1;
    for (int i = 0; i < nb; ++i)
      if (split_fits(M, N, K, bns[i], forced > 0 ? forced : sms, ctas, L))
        return plan_split(M, N, K, bns[i], ctas, L);
    return best;  // grid == 0: not possible (rejected by check_problem)
  }
  if (!(flags & (NVFP4DG_FLAG_NO_SPLITK | NVFP4DG_FLAG_FORCE_STREAMK)) &&
      forced == 0) {
    for (int c = 0; c < nc; ++c) {
      for (int i = 0; i < nb; ++i) {
        if (!split_fits(M, N, K, bns[i], sms, ctas_opts[c], L)) continue;
        Plan p = plan_split(M, N, K, bns[i], ctas_opts[c], L);
        const double cost = plan_cost(p);
        if (cost < best_cost) {
          best_cost = cost;
          best = p;
        }
      }
    }
  }
  for (int c = 0; c < nc; ++c) {
    const int ctas = ctas_opts[c];
    // forced grid counts CTAs; pairs use half as many units
    const int cap = std::max(1, (forced > 0 ? forced : sms) / ctas);
    for (int i = 0; i < nb; ++i) {
      for (int sk = force_sk ? 1 : 0; sk < (streamk ? 2 : 1); ++sk) {
        // Stream-K over fewer tiles than units may also run on a smaller
        // grid: fewer contributors per tile, cheaper fixups.
        int caps[6];
        int ncap = 0;
        caps[ncap++] = cap;
        if (sk == 1 && forced == 0) {
          const long long tiles = (long long)L *
                                  ((M + kBM * ctas - 1) / (kBM * ctas)) *
                                  (N / bns[i]);
          for (int f : {2, 3, 4, 6, 8})
            if (tiles * f < cap) caps[ncap++] = static_cast<int>(tiles * f);
        }
        for (int j = 0; j < ncap; ++j) {
          Plan p = plan_for(M, N, K, bns[i], ctas, caps[j], sk == 1, force_sk,
                            L);
          const double cost = plan_cost(p);
          if (cost < best_cost) {
            best_cost = cost;
            best = p;
          }
        }
      }
    }
  }
  return best;
}

// The schedules of recent problems: the cost model weighs a few dozen
// candidate plans (~2 us of host time), which a caller that repeats the same
// shapes (one call per layer and step) should pay once.  Small, direct
// mapped, guarded by g_mu like the other host caches; the flag bits that
// only affect the launch (not the plan) are left out of the key.
struct PlanKey {
  int M, N, K, L, sms;
  unsigned flags;
  bool operator==(const PlanKey& o) const {
    return M == o.M && N == o.N && K == o.K && L == o.L && sms == o.sms &&
           flags == o.flags;
  }
};
constexpr int kPlanCacheSize = 32;
struct PlanCacheEntry {
  bool used;
  PlanKey key;
  Plan plan;
};
PlanCacheEntry g_plan_cache[kPlanCacheSize];

Plan cached_plan(int M, int N, int K, unsigned flags, int sms, int L) {
  constexpr unsigned kLaunchOnly = NVFP4DG_FLAG_SYNC_CHECK | NVFP4DG_FLAG_NO_PDL |
                                   NVFP4DG_FLAG_NO_MERGED_B |
                                   NVFP4DG_FLAG_STATIC_WEIGHTS |
                                   NVFP4DG_FLAG_TEST_SK_TIMEOUT |
                                   NVFP4DG_FLAG_NO_TMA_STORE;
  const PlanKey key{M, N, K, L, sms, flags & ~kLaunchOnly};
  const unsigned h = (static_cast<unsigned>(M) * 2654435761u ^
                      static_cast<unsigned>(N) * 40503u ^
                      static_cast<unsigned>(K) * 97u ^
                      static_cast<unsigned>(L) * 131u ^ key.flags) %
                     kPlanCacheSize;
  PlanCacheEntry& e = g_plan_cache[h];
  if (e.used && e.key == key) return e.plan;
  const Plan plan = choose_plan(M, N, K, key.flags, sms, L);
  e.used = true;
  e.key = key;
  e.plan = plan;
  return plan;
}

int check_problem(const void* A, const void* B1, const void* B2,
                  const void* SFA, const void* SFB1, const void* SFB2,
                  const void* C, int M, int N, int K, int L, unsigned flags,
                  bool device_ptrs = true, bool allow_batch = false) {
  if (M < 0 || N < 0 || K < 0)
    return fail(NVFP4DG_ERR_INVALID, "M, N, K must be non-negative");
  if (L < 1 || (L != 1 && !allow_batch))
    return fail(NVFP4DG_ERR_INVALID,
                allow_batch ? "L must be >= 1"
                            : "L must be 1 for this entry point (batched "
                              "problems go through nvfp4_dual_gemm_run)");
  if ((long long)L * ((M + 255) / 256) * (N / 64) >= (1ll << 30))
    return fail(NVFP4DG_ERR_INVALID, "too many tiles (L * M * N too large)");
  if (N % 64 != 0)
    return fail(NVFP4DG_ERR_INVALID, "N must be a multiple of 64");
  if (K % 256 != 0)
    return fail(NVFP4DG_ERR_INVALID, "K must be a multiple of 256");
  if ((flags & NVFP4DG_FLAG_BN128) && N % 128 != 0)
    return fail(NVFP4DG_ERR_INVALID, "BN=128 forced but N % 128 != 0");
  if ((flags & NVFP4DG_FLAG_BN64) && (flags & NVFP4DG_FLAG_BN128))
    return fail(NVFP4DG_ERR_INVALID, "BN64 and BN128 flags are exclusive");
  if ((flags & NVFP4DG_FLAG_FORCE_STREAMK) && (flags & NVFP4DG_FLAG_NO_STREAMK))
    return fail(NVFP4DG_ERR_INVALID,
                "FORCE_STREAMK and NO_STREAMK flags are exclusive");
  if ((flags & NVFP4DG_FLAG_PAIR) && (flags & NVFP4DG_FLAG_NO_PAIR))
    return fail(NVFP4DG_ERR_INVALID, "PAIR and NO_PAIR flags are exclusive");
  if ((flags & NVFP4DG_FLAG_SPLITK) &&
      (flags & (NVFP4DG_FLAG_NO_SPLITK | NVFP4DG_FLAG_FORCE_STREAMK)))
    return fail(NVFP4DG_ERR_INVALID,
                "SPLITK excludes NO_SPLITK and FORCE_STREAMK");
  if (M == 0 || N == 0) return NVFP4DG_OK;
  const void* ptrs[7] = {A, B1, B2, SFA, SFB1, SFB2, C};
  const char* names[7] = {"A", "B1", "B2", "SFA", "SFB1", "SFB2", "C"};
  for (int i = 0; i < 7; ++i) {
    if (K == 0 && i < 6) continue;
    if (ptrs[i] == nullptr)
      return fail(NVFP4DG_ERR_INVALID, std::string(names[i]) + " is NULL");
    if (device_ptrs && reinterpret_cast<uintptr_t>(ptrs[i]) % 16 != 0)
      return fail(NVFP4DG_ERR_ALIGN,
                  std::string(names[i]) + " is not 16-byte aligned");
  }
  return NVFP4DG_OK;
}

template <int BN, bool PAIR>
int launch(const Plan& plan, DevInfo& dev, int devid, const void* A,
           const void* B1, const void* B2, const void* SFA, const void* SFB1,
           const void* SFB2, void* C, int M, int N, int K, void* ws,
           unsigned flags, cudaStream_t stream, void* cq = nullptr,
           void* sfc = nullptr, const GroupTable* groups = nullptr) {
  constexpr int kSmem = PAIR ? PairCfg<BN>::kSmemBytes : Cfg<BN>::kSmemBytes;
  auto kernel = PAIR ? dual_gemm_pair_kernel<BN> : dual_gemm_kernel<BN>;
  bool& attr = PAIR ? (BN == 64 ? dev.attr64p : dev.attr128p)
                    : (BN == 64 ? dev.attr64 : dev.attr128);
  if (!attr) {
    cudaError_t e = cudaFuncSetAttribute(
        kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem);
    if (e != cudaSuccess) return cuda_fail(e, "cudaFuncSetAttribute");
    attr = true;
  }
  CUtensorMap ta, tb1, tb2, tc;
  std::memset(&tc, 0, sizeof(tc));
  int rc;
  // The pair kernel copies with 2-D maps; the 1-SM kernel with 3-D ones,
  // both weight tiles of a K block in one copy when a single map can cover
  // B1 and B2.  Batched problems (L > 1) use 3-D maps in both kernels, the
  // batch being the third coordinate, and separate B1 / B2 maps.
  // Grouped problems: A is one matrix of M (all groups') rows, the weights
  // one batch per group.
  const int a_layers = groups ? 1 : plan.L;
  const int b_layers = groups ? groups->count : plan.L;
  const bool maps3d = !PAIR || a_layers > 1 || b_layers > 1;
  const int rank = maps3d ? 3 : 2;
  if ((rc = tensor_map(A, M, K / 2, kBM, devid, &ta, rank, a_layers)))
    return rc;
  const bool merged = !PAIR && b_layers == 1 &&
                      !(flags & NVFP4DG_FLAG_NO_MERGED_B) &&
                      b_pair_map(B1, B2, N, K / 2, BN, devid, &tb1);
  if (merged) {
    tb2 = tb1;
  } else {
    if ((rc = tensor_map(B1, N, K / 2, BN, devid, &tb1, rank, b_layers)))
      return rc;
    if ((rc = tensor_map(B2, N, K / 2, BN, devid, &tb2, rank, b_layers)))
      return rc;
  }
  KParams kp;
  kp.plan = plan;
  kp.M = M;
  kp.N = N;
  kp.K = K;
  kp.sfa_batch = blocked_scale_bytes(M, K);
  kp.sfb_batch = blocked_scale_bytes(N, K);
  kp.sfc_batch = blocked_scale_bytes(M, N);
  kp.sfa = static_cast<const uint8_t*>(SFA);
  kp.sfb1 = static_cast<const uint8_t*>(SFB1);
  kp.sfb2 = static_cast<const uint8_t*>(SFB2);
  kp.C = static_cast<__half*>(C);
  kp.cq = static_cast<uint8_t*>(cq);
  kp.sfc = static_cast<uint8_t*>(sfc);
  kp.counters = static_cast<int*>(ws);
  kp.partials = ws ? reinterpret_cast<float*>(static_cast<uint8_t*>(ws) +
                                              workspace_partials_offset(plan))
                   : nullptr;
  kp.err = dev.err;
  kp.b_merged = merged ? 1 : 0;
  kp.static_weights = (flags & NVFP4DG_FLAG_STATIC_WEIGHTS) ? 1 : 0;
  kp.maps3d = maps3d ? 1 : 0;
  // fp16 C through TMA stores (pair kernel, BN = 128, not grouped, unless
  // NVFP4DG_FLAG_NO_TMA_STORE): a byte view of C, rows of 2N bytes,
  // 128-byte x 128-row boxes (64 columns)
  kp.c_tma = 0;
  kp.c_layers = plan.L;
  if (PAIR && BN == 128 && C != nullptr && groups == nullptr &&
      !(flags & NVFP4DG_FLAG_NO_TMA_STORE)) {
    if ((rc = tensor_map(C, M, 2ll * N, kBM, devid, &tc,
                         plan.L > 1 ? 3 : 2, plan.L)))
      return rc;
    kp.c_tma = 1;
  }
  const bool expire = (flags & NVFP4DG_FLAG_TEST_SK_TIMEOUT) != 0;
  kp.sk_extra = expire ? 1 : 0;
  kp.sk_wait_limit = expire ? kTestWaitLimitCycles : kWaitLimitCycles;
  if (groups) {
    kp.groups = *groups;
  } else {
    kp.groups.count = 0;
  }
  // Programmatic dependent launch lets this grid be scheduled while the
  // previous one in the stream finishes (the kernel waits for it before its
  // first global access); clusters as set below.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(plan.grid * plan.ctas, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = stream;
  cudaLaunchAttribute attrs[2];
  unsigned na = 0;
  if (!(flags & NVFP4DG_FLAG_NO_PDL)) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  // clusters: a 2-SM pair (2), a split-K pair of CTAs (2) or of 2-SM pairs
  // (4)
  const int cluster = (PAIR ? 2 : 1) * (plan.split == 2 ? 2 : 1);
  if (cluster > 1) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = cluster;
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, ta, tb1, tb2, tc, kp);
  if (e != cudaSuccess) return cuda_fail(e, "dual_gemm_kernel launch");
  return NVFP4DG_OK;
}

int read_status(int dev, unsigned* word) {
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(dev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  DevInfo* d = nullptr;
  int rc = device_info(dev, &d);
  if (rc == NVFP4DG_OK) {
    unsigned v = 0;
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(&v, g_err_word, sizeof(v));
    const unsigned zero = 0;
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_err_word, &zero, sizeof(zero));
    if (e != cudaSuccess) rc = cuda_fail(e, "reading the device error word");
    *word = v;
  }
  cudaSetDevice(prev);
  return rc;
}

// Grouped problems: the schedule over all groups' tiles (m fastest within a
// group, then n, then the group) and the kernels' group table.  Cluster
// split-K is not used; among 2-SM pair and single-CTA tiles, each tile width
// and stream-K or not, the plan with the least modelled cost is taken, the
// m tiles of all groups counting as the rows of one problem.
Plan choose_plan_grouped(const int* rows, const int* row0, int G, int N,
                         int K, unsigned flags, int sms, GroupTable* table) {
  Plan best{};
  double best_cost = 1e300;
  for (int ctas = 2; ctas >= 1; --ctas) {
    if (ctas == 2 && (flags & NVFP4DG_FLAG_NO_PAIR)) continue;
    if (ctas == 1 && (flags & NVFP4DG_FLAG_PAIR)) continue;
    long long mt = 0;
    for (int g = 0; g < G; ++g)
      mt += (rows[g] + kBM * ctas - 1) / (kBM * ctas);
    if (mt == 0) continue;
    const unsigned f = (flags & ~(NVFP4DG_FLAG_PAIR | NVFP4DG_FLAG_NO_PAIR)) |
                       NVFP4DG_FLAG_NO_SPLITK |
                       (ctas == 2 ? NVFP4DG_FLAG_PAIR : NVFP4DG_FLAG_NO_PAIR);
    const Plan p = choose_plan(static_cast<int>(mt * kBM * ctas), N, K, f, sms);
    if (p.grid == 0) continue;
    const double c = plan_cost(p);
    if (c < best_cost) {
      best_cost = c;
      best = p;
    }
  }
  if (best.grid == 0) return best;
  table->count = G;
  int t = 0;
  for (int g = 0; g < G; ++g) {
    table->tile0[g] = t;
    table->row0[g] = row0[g];
    table->rows[g] = rows[g];
    t += (rows[g] + kBM * best.ctas - 1) / (kBM * best.ctas) * best.n_tiles;
  }
  table->tile0[G] = t;
  return best;
}

// `cq` / `sfc` not null: NVFP4 output (codes and blocked scales) instead of
// the fp16 C, which is then unused (nvfp4_dual_gemm_run_nvfp4_out).
// `G` > 0: grouped problems (nvfp4_dual_gemm_run_grouped); M is then the row
// count of A and C over all groups, L is 1, and `group_rows` / `group_row0`
// give each group's rows (validated by the caller).
int run_impl(const void* A, const void* B1, const void* B2, const void* SFA,
             const void* SFB1, const void* SFB2, void* C, int M, int N, int K,
             int L, unsigned flags, void* ws, size_t ws_bytes, bool own_ws,
             void* stream_ptr, void* cq = nullptr, void* sfc = nullptr,
             const int* group_rows = nullptr, const int* group_row0 = nullptr,
             int G = 0) {
  g_last_error.clear();
  const bool q_out = cq != nullptr || sfc != nullptr;
  int rc = check_problem(A, B1, B2, SFA, SFB1, SFB2, q_out ? cq : C, M, N, K,
                         L, flags, true, /*allow_batch=*/true);
  if (rc) return rc;
  if (q_out && M > 0 && N > 0) {
    if (sfc == nullptr) return fail(NVFP4DG_ERR_INVALID, "SFC is NULL");
    if (reinterpret_cast<uintptr_t>(sfc) % 16 != 0)
      return fail(NVFP4DG_ERR_ALIGN, "SFC is not 16-byte aligned");
  }
  if (M == 0 || N == 0) return NVFP4DG_OK;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (K == 0) {  // empty sums: silu(0) * 0 = 0
    cudaError_t e;
    if (q_out) {
      e = cudaMemsetAsync(cq, 0, (size_t)L * M * (N / 2), stream);
      if (e == cudaSuccess)
        e = cudaMemsetAsync(sfc, 0, (size_t)L * blocked_scale_bytes(M, N),
                            stream);
    } else {
      e = cudaMemsetAsync(C, 0, (size_t)L * M * N * sizeof(__half), stream);
    }
    return e == cudaSuccess ? NVFP4DG_OK : cuda_fail(e, "cudaMemsetAsync");
  }
  if (q_out) C = nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  int devid = 0;
  cudaError_t e = cudaGetDevice(&devid);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  DevInfo* dev = nullptr;
  if ((rc = device_info(devid, &dev))) return rc;
  GroupTable table;
  table.count = 0;
  const GroupTable* groups = nullptr;
  Plan plan;
  if (G > 0) {
    plan = choose_plan_grouped(group_rows, group_row0, G, N, K, flags,
                               dev->sms, &table);
    if (plan.grid == 0) return NVFP4DG_OK;  // every group is empty
    groups = &table;
  } else {
    plan = cached_plan(M, N, K, flags, dev->sms, L);
  }
  if (plan.grid == 0)
    return fail(NVFP4DG_ERR_UNSUPPORTED,
                "cluster split-K needs 2 x tiles x CTAs per tile <= SMs and K >= 512");
  const size_t need = static_cast<size_t>(workspace_bytes(plan));
  if (own_ws && need > 0) {
    WsEntry& ent = g_ws[{devid, stream_ptr}];
    if (ent.bytes < need) {
      if (ent.ptr) {
        cudaStreamSynchronize(stream);
        cudaFree(ent.ptr);
        ent.ptr = nullptr;
        ent.bytes = 0;
      }
      void* p = nullptr;
      if ((e = cudaMalloc(&p, need)) != cudaSuccess)
        return cuda_fail(e, "cudaMalloc(workspace)");
      if ((e = cudaMemsetAsync(p, 0, need, stream)) != cudaSuccess)
        return cuda_fail(e, "cudaMemsetAsync(workspace)");
      ent.ptr = p;
      ent.bytes = need;
    }
    ws = ent.ptr;
    ws_bytes = ent.bytes;
  }
  if (need > 0) {
    if (ws == nullptr || ws_bytes < need)
      return fail(NVFP4DG_ERR_WORKSPACE,
                  "workspace of " + std::to_string(need) +
                      " bytes required, got " + std::to_string(ws_bytes));
    if (reinterpret_cast<uintptr_t>(ws) % 256 != 0)
      return fail(NVFP4DG_ERR_ALIGN, "workspace is not 256-byte aligned");
  } else {
    ws = nullptr;
  }
  if (plan.ctas == 2 && plan.bn == 128)
    rc = launch<128, true>(plan, *dev, devid, A, B1, B2, SFA, SFB1, SFB2, C, M,
                           N, K, ws, flags, stream, cq, sfc,
                           groups);
  else if (plan.ctas == 2)
    rc = launch<64, true>(plan, *dev, devid, A, B1, B2, SFA, SFB1, SFB2, C, M,
                          N, K, ws, flags, stream, cq, sfc,
                           groups);
  else if (plan.bn == 128)
    rc = launch<128, false>(plan, *dev, devid, A, B1, B2, SFA, SFB1, SFB2, C,
                            M, N, K, ws, flags, stream, cq, sfc,
                           groups);
  else
    rc = launch<64, false>(plan, *dev, devid, A, B1, B2, SFA, SFB1, SFB2, C,
                           M, N, K, ws, flags, stream, cq, sfc,
                           groups);
  if (rc) return rc;
  if (flags & NVFP4DG_FLAG_SYNC_CHECK) {
    unsigned word = 0;
    if ((e = cudaStreamSynchronize(stream)) != cudaSuccess)
      return cuda_fail(e, "cudaStreamSynchronize");
    if ((e = cudaMemcpyFromSymbol(&word, g_err_word, sizeof(word))) !=
        cudaSuccess)
      return cuda_fail(e, "cudaMemcpyFromSymbol");
    if (word != 0) {
      const unsigned zero = 0;
      cudaMemcpyToSymbol(g_err_word, &zero, sizeof(zero));
      // a stream-K owner that gave up left its tile counter behind: clear
      // the counters of the library's own workspace for the next call (a
      // caller-owned workspace must be zero-filled again by the caller)
      if (own_ws && ws != nullptr)
        cudaMemsetAsync(ws, 0, static_cast<size_t>(kCounterBytes), stream);
      return fail(NVFP4DG_ERR_DEVICE,
                  "kernel wait timed out (device error word " +
                      std::to_string(word) + ")");
    }
  }
  return NVFP4DG_OK;
}

// Device address of g_noalloc_scratch, looked up once per device with that
// device current (the symbol name itself is not a device address on the
// host).
std::map<int, void*> g_noalloc_ptr;

int noalloc_scratch(int devid, void** out) {
  auto it = g_noalloc_ptr.find(devid);
  if (it != g_noalloc_ptr.end()) {
    *out = it->second;
    return NVFP4DG_OK;
  }
  void* ptr = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
  if (e != cudaSuccess || ptr == nullptr)
    return cuda_fail(e, "cudaGetSymbolAddress(no-allocation scratch)");
  g_noalloc_ptr[devid] = ptr;
  *out = ptr;
  return NVFP4DG_OK;
}

// ---------------------------------------------------------------------------
// Host-buffer pipeline.  The weights are uploaded in slabs of whole 128-row
// groups of B1/B2 (a slab of the blocked scales is then a contiguous run of
// atoms), each slab's kernel starts as soon as its slab has landed, and each
// slab of C goes back to the host while the next slabs upload: the upload
// (host -> device), the kernels and the download (device -> host, the other
// direction of the link) overlap instead of running back to back.
// ---------------------------------------------------------------------------
constexpr int kMaxSlabs = 16;

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

size_t blocked_bytes(int rows, int K) {
  return static_cast<size_t>((rows + 127) / 128) * (K / 64) * 512;
}

// Device staging buffer: full-size copies of the six inputs, then C stored
// slab by slab (slab j as a dense [M, w_j] block at M * n0_j halves).
struct Staging {
  size_t a, sfa, b1, b2, sfb1, sfb2, c, total;
};

Staging staging_layout(int M, int N, int K) {
  Staging s;
  size_t off = 0;
  s.a = off;
  off += align256(static_cast<size_t>(M) * (K / 2));
  s.sfa = off;
  off += align256(blocked_bytes(M, K));
  s.b1 = off;
  off += align256(static_cast<size_t>(N) * (K / 2));
  s.b2 = off;
  off += align256(static_cast<size_t>(N) * (K / 2));
  s.sfb1 = off;
  off += align256(blocked_bytes(N, K));
  s.sfb2 = off;
  off += align256(blocked_bytes(N, K));
  s.c = off;
  off += align256(static_cast<size_t>(M) * N * sizeof(__half));
  s.total = off;
  return s;
}

// Rows per slab for `req` slabs, rounded up to whole 128-row groups.
int slab_rows_for(int N, int req) {
  const int groups = (N + 127) / 128;
  const int s = std::max(1, std::min({req, kMaxSlabs, groups}));
  return (groups + s - 1) / s * 128;
}

// Modelled time (us) of the host-buffer pipeline with `rows`-row slabs,
// fitted to B200 measurements over PCIe 5: ~54 GB/s up and ~57 GB/s down,
// the two directions overlapping; ~5 us per copy that back-to-back copies do
// not hide (issuing them from more streams does not help); ~12 ns per row
// when a slab of C is a strided (2-D) copy.  Upload of A and its scales,
// then per slab 4 uploads (B1, B2 and their scales); each slab's kernel
// (~4 PFLOP/s plus a 6 us floor) after its uploads; each slab of C
// downloaded after its kernel, behind the previous download.
double host_pipeline_us(int M, int N, int K, int rows) {
  const double bw_up = 54e3, bw_down = 57e3;  // bytes per us
  const double per_copy = 5.0, per_row_2d = 0.012;
  const double a_bytes = (double)M * (K / 2) + (double)blocked_bytes(M, K);
  double up = a_bytes / bw_up + 2 * per_copy;
  double down = 0;
  for (int n0 = 0; n0 < N; n0 += rows) {
    const int w = std::min(rows, N - n0);
    const double b_bytes = 2.0 * w * (K / 2) + 2.0 * blocked_bytes(w, K);
    up += b_bytes / bw_up + 4 * per_copy;
    const double kernel = 6.0 + 4.0 * M * (double)w * K / 4e9;
    down = std::max(down, up + kernel) + (double)M * w * 2 / bw_down +
           per_copy + (w < N ? per_row_2d * M : 0.0);
  }
  return down;
}

// Slab rows: `req` slabs when given, else the count with the least modelled
// time, preferring fewer slabs unless more save at least 2 %.
int host_slab_rows(int M, int N, int K, int req) {
  const int groups = (N + 127) / 128;
  if (groups == 0) return 128;
  if (req > 0) return slab_rows_for(N, req);
  int best = slab_rows_for(N, 1);
  double best_t = host_pipeline_us(M, N, K, best);
  for (int s = 2; s <= std::min(kMaxSlabs, groups); ++s) {
    const int rows = slab_rows_for(N, s);
    const double t = host_pipeline_us(M, N, K, rows);
    if (t < 0.98 * best_t) {
      best = rows;
      best_t = t;
    }
  }
  return best;
}

struct HostPipe {
  cudaStream_t up = nullptr;    // host -> device copies
  cudaStream_t down = nullptr;  // device -> host copies
  cudaEvent_t start = nullptr, up_done = nullptr, down_done = nullptr;
  cudaEvent_t landed[kMaxSlabs] = {};
  cudaEvent_t computed[kMaxSlabs] = {};
};
std::map<int, HostPipe> g_pipe;
std::mutex g_pipe_mu;

int host_pipe(int devid, HostPipe** out) {
  HostPipe& p = g_pipe[devid];
  if (p.up == nullptr) {
    cudaError_t e;
    const unsigned ev = cudaEventDisableTiming;
    if ((e = cudaStreamCreateWithFlags(&p.up, cudaStreamNonBlocking)) ||
        (e = cudaStreamCreateWithFlags(&p.down, cudaStreamNonBlocking)) ||
        (e = cudaEventCreateWithFlags(&p.start, ev)) ||
        (e = cudaEventCreateWithFlags(&p.up_done, ev)) ||
        (e = cudaEventCreateWithFlags(&p.down_done, ev)))
      return cuda_fail(e, "creating the host-pipeline streams");
    for (int j = 0; j < kMaxSlabs; ++j)
      if ((e = cudaEventCreateWithFlags(&p.landed[j], ev)) ||
          (e = cudaEventCreateWithFlags(&p.computed[j], ev)))
        return cuda_fail(e, "creating the host-pipeline events");
  }
  *out = &p;
  return NVFP4DG_OK;
}

int copy_up(void* dst, const void* src, size_t bytes, cudaStream_t s) {
  if (bytes == 0) return NVFP4DG_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, s);
  return e == cudaSuccess ? NVFP4DG_OK : cuda_fail(e, "upload");
}

int run_host_impl(const void* A, const void* B1, const void* B2,
                  const void* SFA, const void* SFB1, const void* SFB2, void* C,
                  int M, int N, int K, int L, unsigned flags, int slabs,
                  void* staging, size_t staging_bytes, void* stream_ptr) {
  g_last_error.clear();
  if (slabs < 0 || slabs > kMaxSlabs)
    return fail(NVFP4DG_ERR_INVALID,
                "slabs must be 0 (automatic) to " + std::to_string(kMaxSlabs));
  // The staging buffer's weights are rewritten by every call's uploads, so
  // the weights may never be read before the dependency wait here.
  flags &= ~NVFP4DG_FLAG_STATIC_WEIGHTS;
  // Host buffers need no alignment (the copies take any address).
  int rc = check_problem(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, L, flags,
                         false);
  if (rc) return rc;
  if (M == 0 || N == 0) return NVFP4DG_OK;
  const Staging lay = staging_layout(M, N, K);
  if (staging == nullptr || staging_bytes < lay.total)
    return fail(NVFP4DG_ERR_WORKSPACE,
                "staging buffer of " + std::to_string(lay.total) +
                    " bytes required, got " + std::to_string(staging_bytes));
  if (reinterpret_cast<uintptr_t>(staging) % 256 != 0)
    return fail(NVFP4DG_ERR_ALIGN, "staging buffer is not 256-byte aligned");
  const int rows = host_slab_rows(M, N, K, slabs);
  const int nslab = (N + rows - 1) / rows;
  // Every slab's schedule must exist before anything is enqueued.
  if (K > 0) {
    int devid = 0;
    cudaError_t e = cudaGetDevice(&devid);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    DevInfo* dev = nullptr;
    {
      std::lock_guard<std::mutex> lock(g_mu);
      if ((rc = device_info(devid, &dev))) return rc;
    }
    for (int j = 0; j < nslab; ++j) {
      const int w = std::min(rows, N - j * rows);
      if (choose_plan(M, w, K, flags, dev->sms).grid == 0)
        return fail(NVFP4DG_ERR_UNSUPPORTED,
                    "cluster split-K needs 2 x tiles x CTAs per tile <= SMs and K >= 512 "
                    "(slab of " + std::to_string(w) + " columns)");
    }
  }
  std::lock_guard<std::mutex> lock(g_pipe_mu);
  int devid = 0;
  cudaError_t e = cudaGetDevice(&devid);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  HostPipe* pp = nullptr;
  if ((rc = host_pipe(devid, &pp))) return rc;
  HostPipe& p = *pp;
  cudaStream_t s0 = static_cast<cudaStream_t>(stream_ptr);
  uint8_t* st = static_cast<uint8_t*>(staging);
  const size_t row_b = static_cast<size_t>(K) / 2;
  const size_t atom_row = static_cast<size_t>(K / 64) * 512;  // per 128 rows
  if (nslab == 1) {
    // Nothing to overlap: upload, kernel and download in order on the
    // caller's stream, without the copy streams' event hand-offs (a few us
    // each on a call that the PCIe transfers already bound).
    const size_t n_sf = static_cast<size_t>(blocked_bytes(N, K));
    rc = copy_up(st + lay.a, A, M * row_b, s0);
    if (!rc) rc = copy_up(st + lay.sfa, SFA, blocked_bytes(M, K), s0);
    if (!rc) rc = copy_up(st + lay.b1, B1, N * row_b, s0);
    if (!rc) rc = copy_up(st + lay.b2, B2, N * row_b, s0);
    if (!rc) rc = copy_up(st + lay.sfb1, SFB1, n_sf, s0);
    if (!rc) rc = copy_up(st + lay.sfb2, SFB2, n_sf, s0);
    __half* cs = reinterpret_cast<__half*>(st + lay.c);
    if (!rc)
      rc = run_impl(st + lay.a, st + lay.b1, st + lay.b2, st + lay.sfa,
                    st + lay.sfb1, st + lay.sfb2, cs, M, N, K, 1, flags,
                    nullptr, 0, true, s0);
    if (!rc &&
        (e = cudaMemcpyAsync(C, cs, static_cast<size_t>(M) * N * sizeof(__half),
                             cudaMemcpyDeviceToHost, s0)))
      rc = cuda_fail(e, "download");
    return rc;
  }
  // Uploads start once everything before this call on the caller's stream
  // (an earlier call still reading the staging buffer) is done.
  if ((e = cudaEventRecord(p.start, s0)) ||
      (e = cudaStreamWaitEvent(p.up, p.start, 0)))
    return cuda_fail(e, "ordering the upload stream");
  rc = copy_up(st + lay.a, A, M * row_b, p.up);
  if (!rc) rc = copy_up(st + lay.sfa, SFA, blocked_bytes(M, K), p.up);
  for (int j = 0; j < nslab && !rc; ++j) {
    const size_t n0 = static_cast<size_t>(j) * rows;
    const size_t n1 = std::min<size_t>(N, n0 + rows);
    rc = copy_up(st + lay.b1 + n0 * row_b, static_cast<const uint8_t*>(B1) +
                 n0 * row_b, (n1 - n0) * row_b, p.up);
    if (!rc)
      rc = copy_up(st + lay.b2 + n0 * row_b,
                   static_cast<const uint8_t*>(B2) + n0 * row_b,
                   (n1 - n0) * row_b, p.up);
    const size_t g0 = n0 / 128, g1 = (n1 + 127) / 128;
    if (!rc)
      rc = copy_up(st + lay.sfb1 + g0 * atom_row,
                   static_cast<const uint8_t*>(SFB1) + g0 * atom_row,
                   (g1 - g0) * atom_row, p.up);
    if (!rc)
      rc = copy_up(st + lay.sfb2 + g0 * atom_row,
                   static_cast<const uint8_t*>(SFB2) + g0 * atom_row,
                   (g1 - g0) * atom_row, p.up);
    if (!rc && (e = cudaEventRecord(p.landed[j], p.up)))
      rc = cuda_fail(e, "recording an upload event");
  }
  // Kernels on the caller's stream, one per slab, each after its slab lands;
  // downloads on their own stream, each after its slab's kernel.
  for (int j = 0; j < nslab && !rc; ++j) {
    const size_t n0 = static_cast<size_t>(j) * rows;
    const int w = std::min(rows, N - j * rows);
    if ((e = cudaStreamWaitEvent(s0, p.landed[j], 0))) {
      rc = cuda_fail(e, "waiting for an upload");
      break;
    }
    __half* cs = reinterpret_cast<__half*>(st + lay.c) + n0 * M;
    rc = run_impl(st + lay.a, st + lay.b1 + n0 * row_b, st + lay.b2 + n0 * row_b,
                  st + lay.sfa, st + lay.sfb1 + (n0 / 128) * atom_row,
                  st + lay.sfb2 + (n0 / 128) * atom_row, cs, M, w, K, 1, flags,
                  nullptr, 0, true, s0);
    if (rc) break;
    if ((e = cudaEventRecord(p.computed[j], s0)) ||
        (e = cudaStreamWaitEvent(p.down, p.computed[j], 0))) {
      rc = cuda_fail(e, "ordering the download stream");
      break;
    }
    const size_t pitch = static_cast<size_t>(N) * sizeof(__half);
    const size_t width = static_cast<size_t>(w) * sizeof(__half);
    if ((e = cudaMemcpy2DAsync(static_cast<uint8_t*>(C) + n0 * sizeof(__half),
                               pitch, cs, width, width, M,
                               cudaMemcpyDeviceToHost, p.down))) {
      rc = cuda_fail(e, "download");
      break;
    }
  }
  // The caller's stream completes only after both copy streams have, also
  // when an error stopped the loop part-way.
  cudaError_t e1 = cudaEventRecord(p.up_done, p.up);
  if (!e1) e1 = cudaEventRecord(p.down_done, p.down);
  if (!e1) e1 = cudaStreamWaitEvent(s0, p.up_done, 0);
  if (!e1) e1 = cudaStreamWaitEvent(s0, p.down_done, 0);
  if (e1 && !rc) rc = cuda_fail(e1, "joining the copy streams");
  return rc;
}

}  // namespace

// ===========================================================================
// C ABI
// ===========================================================================
extern "C" {

int nvfp4_dual_gemm_run(const void* A, const void* B1, const void* B2,
                        const void* SFA, const void* SFB1, const void* SFB2,
                        void* C, int M, int N, int K, int L, unsigned flags,
                        void* stream) {
  return run_impl(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, L, flags, nullptr, 0,
                  true, stream);
}

int nvfp4_dual_gemm_run_grouped(const void* A, const void* B1,
                                const void* B2, const void* SFA,
                                const void* SFB1, const void* SFB2, void* C,
                                const int* group_rows, const int* group_row0,
                                int groups, int N, int K, unsigned flags,
                                void* workspace, size_t workspace_bytes,
                                void* stream) {
  g_last_error.clear();
  if (groups < 1 || groups > kMaxGroups)
    return fail(NVFP4DG_ERR_INVALID,
                "groups must be 1.." + std::to_string(kMaxGroups));
  if (group_rows == nullptr || group_row0 == nullptr)
    return fail(NVFP4DG_ERR_INVALID, "group_rows and group_row0 are required");
  if (flags & NVFP4DG_FLAG_SPLITK)
    return fail(NVFP4DG_ERR_INVALID,
                "cluster split-K is not available for grouped problems");
  long long next = 0, R = 0;
  for (int g = 0; g < groups; ++g) {
    const long long rows = group_rows[g], r0 = group_row0[g];
    if (rows < 0 || r0 < 0 || r0 % kBM != 0)
      return fail(NVFP4DG_ERR_INVALID,
                  "group " + std::to_string(g) +
                      ": rows must be >= 0 and the first row a multiple of "
                      "128");
    if (r0 < next)
      return fail(NVFP4DG_ERR_INVALID,
                  "group " + std::to_string(g) +
                      " overlaps the previous one (each group's rows, rounded "
                      "up to 128, must end before the next group starts)");
    next = r0 + (rows + kBM - 1) / kBM * kBM;
    if (rows > 0) R = std::max(R, r0 + rows);
  }
  if (next >= (1ll << 31))
    return fail(NVFP4DG_ERR_INVALID, "too many rows");
  const int M = static_cast<int>(R);
  if (K == 0 && M > 0 && N > 0) {  // empty sums: each group's rows are 0
    int rc = check_problem(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, 1, flags);
    if (rc) return rc;
    for (int g = 0; g < groups; ++g) {
      if (group_rows[g] == 0) continue;
      cudaError_t e = cudaMemsetAsync(
          static_cast<__half*>(C) + (size_t)group_row0[g] * N, 0,
          (size_t)group_rows[g] * N * sizeof(__half),
          static_cast<cudaStream_t>(stream));
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync");
    }
    return NVFP4DG_OK;
  }
  return run_impl(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, 1,
                  flags | NVFP4DG_FLAG_NO_SPLITK, workspace, workspace_bytes,
                  workspace == nullptr, stream, nullptr, nullptr, group_rows,
                  group_row0, groups);
}

size_t nvfp4_dual_gemm_grouped_workspace_size(const int* group_rows,
                                              int groups, int N, int K,
                                              unsigned flags) {
  g_last_error.clear();
  if (group_rows == nullptr || groups < 1 || groups > kMaxGroups || N <= 0 ||
      K <= 0 || N % 64 || K % 256)
    return 0;
  int devid = 0;
  if (cudaGetDevice(&devid) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(g_mu);
  DevInfo* dev = nullptr;
  if (device_info(devid, &dev)) return 0;
  std::vector<int> row0(groups, 0);
  GroupTable table;
  const Plan p = choose_plan_grouped(group_rows, row0.data(), groups, N, K,
                                     flags | NVFP4DG_FLAG_NO_SPLITK, dev->sms,
                                     &table);
  return p.grid == 0 ? 0 : static_cast<size_t>(workspace_bytes(p));
}

int nvfp4_dual_gemm_run_nvfp4_out(const void* A, const void* B1,
                                  const void* B2, const void* SFA,
                                  const void* SFB1, const void* SFB2,
                                  void* Cq, void* SFC, int M, int N, int K,
                                  int L, unsigned flags, void* stream) {
  if (Cq == nullptr && M > 0 && N > 0) {
    g_last_error.clear();
    return fail(NVFP4DG_ERR_INVALID, "Cq is NULL");
  }
  return run_impl(A, B1, B2, SFA, SFB1, SFB2, nullptr, M, N, K, L, flags,
                  nullptr, 0, true, stream, Cq, SFC);
}

size_t nvfp4_dual_gemm_host_staging_size(int M, int N, int K, int L) {
  g_last_error.clear();
  if (M < 0 || N < 0 || K < 0 || L != 1 || N % 64 != 0 || K % 256 != 0) {
    fail(NVFP4DG_ERR_INVALID, "invalid problem shape");
    return 0;
  }
  if (M == 0 || N == 0) return 0;
  return staging_layout(M, N, K).total;
}

int nvfp4_dual_gemm_host_slabs(int M, int N, int K, int slabs) {
  if (M < 0 || N <= 0 || K < 0 || slabs < 0 || slabs > kMaxSlabs) return 0;
  const int rows = host_slab_rows(M, N, K, slabs);
  return (N + rows - 1) / rows;
}

int nvfp4_dual_gemm_run_host(const void* A, const void* B1, const void* B2,
                             const void* SFA, const void* SFB1,
                             const void* SFB2, void* C, int M, int N, int K,
                             int L, unsigned flags, int slabs, void* staging,
                             size_t staging_bytes, void* stream) {
  return run_host_impl(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, L, flags, slabs,
                       staging, staging_bytes, stream);
}

int nvfp4_dual_gemm_run_ws(const void* A, const void* B1, const void* B2,
                           const void* SFA, const void* SFB1, const void* SFB2,
                           void* C, int M, int N, int K, int L, unsigned flags,
                           void* workspace, size_t workspace_bytes,
                           void* stream) {
  return run_impl(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, L, flags, workspace,
                  workspace_bytes, false, stream);
}

int nvfp4_dual_gemm_run_noalloc(const void* A, const void* B1, const void* B2,
                                const void* SFA, const void* SFB1,
                                const void* SFB2, void* C, int M, int N, int K,
                                int L, unsigned flags, void* stream_ptr) {
  g_last_error.clear();
  int rc = check_problem(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, L, flags);
  if (rc) return rc;
  if (M == 0 || N == 0 || K == 0)  // nothing needs scratch
    return run_impl(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, L, flags, nullptr,
                    0, false, stream_ptr);
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_mu);
    int devid = 0;
    cudaError_t e = cudaGetDevice(&devid);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    DevInfo* dev = nullptr;
    if ((rc = device_info(devid, &dev))) return rc;
    if ((rc = noalloc_scratch(devid, &scratch))) return rc;
    // The automatic schedule may split tiles along K over a full grid
    // (stream-K), whose partials can exceed the array; whole tiles need no
    // scratch at all, so fall back to them unless stream-K was forced.
    size_t need = static_cast<size_t>(
        workspace_bytes(cached_plan(M, N, K, flags, dev->sms, 1)));
    if (need > NVFP4DG_NOALLOC_SCRATCH_BYTES &&
        !(flags & NVFP4DG_FLAG_FORCE_STREAMK)) {
      flags |= NVFP4DG_FLAG_NO_STREAMK;
      need = static_cast<size_t>(
          workspace_bytes(cached_plan(M, N, K, flags, dev->sms, 1)));
    }
    if (need > NVFP4DG_NOALLOC_SCRATCH_BYTES)
      return fail(NVFP4DG_ERR_WORKSPACE,
                  "this schedule needs " + std::to_string(need) +
                      " bytes of scratch; nvfp4_dual_gemm_run_noalloc holds "
                      "at most " +
                      std::to_string(NVFP4DG_NOALLOC_SCRATCH_BYTES) +
                      " (use nvfp4_dual_gemm_run_ws or a smaller forced "
                      "grid)");
    if (need > 0) {
      // The array keeps the previous call's contents (a call that timed out
      // may leave counts behind): zero the tile counters.
      e = cudaMemsetAsync(scratch, 0, static_cast<size_t>(kCounterBytes),
                          static_cast<cudaStream_t>(stream_ptr));
      if (e != cudaSuccess) return cuda_fail(e, "cudaMemsetAsync(scratch)");
    }
  }
  return run_impl(A, B1, B2, SFA, SFB1, SFB2, C, M, N, K, L, flags, scratch,
                  NVFP4DG_NOALLOC_SCRATCH_BYTES, false, stream_ptr);
}

size_t nvfp4_dual_gemm_workspace_size(int M, int N, int K, int L,
                                      unsigned flags) {
  g_last_error.clear();
  if (M <= 0 || N <= 0 || K <= 0 || L < 1 || N % 64 || K % 256) return 0;
  int devid = 0;
  if (cudaGetDevice(&devid) != cudaSuccess) return 0;
  std::lock_guard<std::mutex> lock(g_mu);
  DevInfo* dev = nullptr;
  if (device_info(devid, &dev)) return 0;
  return static_cast<size_t>(
      workspace_bytes(cached_plan(M, N, K, flags, dev->sms, L)));
}

int nvfp4_dual_gemm_plan(int M, int N, int K, unsigned flags, int num_sms,
                         int* bn_out, int* ctas_out, int* grid_out,
                         int* dp_tiles_out, int* sk_tiles_out,
                         int* split_out) {
  g_last_error.clear();
  if (M <= 0 || N <= 0 || K <= 0 || N % 64 || K % 256 || num_sms <= 0)
    return fail(NVFP4DG_ERR_INVALID, "invalid problem for planning");
  const Plan p = choose_plan(M, N, K, flags, num_sms);
  if (p.grid == 0)
    return fail(NVFP4DG_ERR_UNSUPPORTED,
                "cluster split-K needs 2 x tiles x CTAs per tile <= SMs and K >= 512");
  if (split_out) *split_out = p.split;
  if (bn_out) *bn_out = p.bn;
  if (ctas_out) *ctas_out = p.ctas;
  if (grid_out) *grid_out = p.grid;
  if (dp_tiles_out) *dp_tiles_out = p.dp_tiles;
  if (sk_tiles_out) *sk_tiles_out = p.num_tiles - p.dp_tiles;
  return NVFP4DG_OK;
}

int nvfp4_dual_gemm_plan_work(int M, int N, int K, unsigned flags, int num_sms,
                              int cta, int* records, int cap) {
  g_last_error.clear();
  if (M <= 0 || N <= 0 || K <= 0 || N % 64 || K % 256 || num_sms <= 0) {
    fail(NVFP4DG_ERR_INVALID, "invalid problem for planning");
    return -1;
  }
  const Plan p = choose_plan(M, N, K, flags, num_sms);
  if (cta < 0 || cta >= p.grid) {
    fail(NVFP4DG_ERR_INVALID, "cta out of range");
    return -1;
  }
  WorkIter it;
  work_begin(p, cta, it);
  Work w;
  int n = 0;
  while (work_next(p, it, w)) {
    if (n < cap && records) {
      records[4 * n + 0] = w.tile;
      records[4 * n + 1] = w.kb0;
      records[4 * n + 2] = w.kb1;
      records[4 * n + 3] = w.slot;
    }
    ++n;
  }
  return n;
}

int nvfp4_quantize_rows(const void* X, int dtype, int rows, int K,
                        long long ldx, void* codes, void* sf_plain,
                        void* sf_blocked, void* stream_ptr) {
  g_last_error.clear();
  if (rows < 0 || K < 0 || K % 64 != 0)
    return fail(NVFP4DG_ERR_INVALID, "rows >= 0 and K % 64 == 0 required");
  if (dtype != NVFP4DG_DTYPE_F32 && dtype != NVFP4DG_DTYPE_F16 &&
      dtype != NVFP4DG_DTYPE_BF16)
    return fail(NVFP4DG_ERR_INVALID, "dtype must be F32, F16 or BF16");
  if (rows == 0 || K == 0) return NVFP4DG_OK;
  if (ldx < K)
    return fail(NVFP4DG_ERR_INVALID, "ldx must be at least K");
  if (!X || !codes || !sf_blocked)
    return fail(NVFP4DG_ERR_INVALID, "X, codes and sf_blocked are required");
  const size_t esize = dtype == NVFP4DG_DTYPE_F32 ? 4 : 2;
  if (reinterpret_cast<uintptr_t>(X) % 16 || (ldx * esize) % 16 ||
      reinterpret_cast<uintptr_t>(codes) % 16 ||
      reinterpret_cast<uintptr_t>(sf_blocked) % 16 ||
      reinterpret_cast<uintptr_t>(sf_plain) % 4)
    return fail(NVFP4DG_ERR_ALIGN,
                "X, its row pitch, codes and sf_blocked must be 16-byte "
                "aligned, sf_plain 4-byte aligned");
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long units =
      ((long long)rows + 127) / 128 * 128 * ((K + 1023) / 1024);
  const int threads = 256;
  const long long want = (units + threads / 32 - 1) / (threads / 32);
  const int blocks = (int)std::min<long long>(want, (long long)sms * 8);
  uint8_t* c8 = static_cast<uint8_t*>(codes);
  uint8_t* p8 = static_cast<uint8_t*>(sf_plain);
  uint8_t* b8 = static_cast<uint8_t*>(sf_blocked);
  if (dtype == NVFP4DG_DTYPE_F32)
    quantize_rows_kernel<float><<<blocks, threads, 0, stream>>>(
        static_cast<const float*>(X), rows, K, ldx, c8, p8, b8);
  else if (dtype == NVFP4DG_DTYPE_F16)
    quantize_rows_kernel<__half><<<blocks, threads, 0, stream>>>(
        static_cast<const __half*>(X), rows, K, ldx, c8, p8, b8);
  else
    quantize_rows_kernel<__nv_bfloat16><<<blocks, threads, 0, stream>>>(
        static_cast<const __nv_bfloat16*>(X), rows, K, ldx, c8, p8, b8);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "quantize_rows_kernel launch");
  return NVFP4DG_OK;
}

int convert_scales(const void* src, void* dst, int rows, int K, long long ld,
                   bool to_blocked, void* stream_ptr) {
  g_last_error.clear();
  if (rows < 0 || K < 0 || K % 64 != 0)
    return fail(NVFP4DG_ERR_INVALID, "rows >= 0 and K % 64 == 0 required");
  if (rows == 0 || K == 0) return NVFP4DG_OK;
  if (ld < K / 16)
    return fail(NVFP4DG_ERR_INVALID, "ld must be at least K / 16 bytes");
  if (!src || !dst) return fail(NVFP4DG_ERR_INVALID, "NULL buffer");
  const void* plain = to_blocked ? src : dst;
  const void* blk = to_blocked ? dst : src;
  if (reinterpret_cast<uintptr_t>(plain) % 4 || ld % 4 ||
      reinterpret_cast<uintptr_t>(blk) % 16)
    return fail(NVFP4DG_ERR_ALIGN,
                "plain scales and their row pitch must be 4-byte aligned, "
                "blocked scales 16-byte aligned");
  const int groups = K / 64;
  const dim3 grid((groups + kCvtGroups - 1) / kCvtGroups, (rows + 127) / 128);
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  if (to_blocked)
    scales_to_blocked_kernel<<<grid, 256, 0, stream>>>(
        static_cast<const uint8_t*>(src), rows, groups, ld,
        static_cast<uint8_t*>(dst));
  else
    scales_from_blocked_kernel<<<grid, 256, 0, stream>>>(
        static_cast<const uint8_t*>(src), rows, groups, ld,
        static_cast<uint8_t*>(dst));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e, "scale layout kernel launch");
  return NVFP4DG_OK;
}

int nvfp4_scales_to_blocked(const void* plain, int rows, int K, long long ld,
                            void* blocked, void* stream) {
  return convert_scales(plain, blocked, rows, K, ld, true, stream);
}

int nvfp4_scales_from_blocked(const void* blocked, int rows, int K,
                              void* plain, long long ld, void* stream) {
  return convert_scales(blocked, plain, rows, K, ld, false, stream);
}

int nvfp4_quantize(const float* X, int rows, int K, void* codes,
                   void* sf_plain, void* sf_blocked, void* stream_ptr) {
  return nvfp4_quantize_rows(X, NVFP4DG_DTYPE_F32, rows, K, K, codes, sf_plain,
                             sf_blocked, stream_ptr);
}

int nvfp4_dual_gemm_device_status(int device, unsigned* word_out) {
  g_last_error.clear();
  if (!word_out) return fail(NVFP4DG_ERR_INVALID, "word_out is NULL");
  std::lock_guard<std::mutex> lock(g_mu);
  return read_status(device, word_out);
}

const char* nvfp4_dual_gemm_last_error(void) { return g_last_error.c_str(); }

#ifdef NVFP4DG_TRACE
// Trace builds only: copy the stamp buffer ([160][8][64] int64) to the host.
NVFP4DG_API int nvfp4_dual_gemm_trace_read(void* host, size_t bytes) {
  if (bytes < sizeof(g_trace)) return NVFP4DG_ERR_INVALID;
  cudaError_t e = cudaMemcpyFromSymbol(host, g_trace, sizeof(g_trace));
  const long long zero[kTraceSlots] = {};
  for (int c = 0; c < kTraceCtas && e == cudaSuccess; ++c)
    for (int r = 0; r < kTraceRoles && e == cudaSuccess; ++r)
      e = cudaMemcpyToSymbol(g_trace, zero, sizeof(zero),
                             ((size_t)c * kTraceRoles + r) * sizeof(zero));
  return e == cudaSuccess ? NVFP4DG_OK : NVFP4DG_ERR_CUDA;
}
#endif

int nvfp4_dual_gemm_version(void) { return 101; }

}  // extern "C"
