// Fused Mamba-3 SISO recurrence on the sm_100 tensor cores: persistent,
// chunk-parallel, warp-specialised.
//
// Work units. A unit is one 64-step chunk c of one (batch b, head h) row. Units
// are numbered chunk-major, u = ((c*ndir + dir)*B + b)*H + h, and handed out in
// chunk-major order by an atomic ticket, so a unit only ever depends on units
// already held by running CTAs: the kernel cannot deadlock, whether or not every
// CTA of the grid is resident. Tickets count only non-empty units (chunks that
// start before their row's length): within chunk c, ticket r is head r % H of the
// (r / H)-th row in order of decreasing length, so no CTA spends an iteration on
// a chunk past its row's end (launches of more than kMapRows rows or kMapChunks
// chunks per row hand out every unit instead and skip the empty ones). A CTA takes at most ceil(non-empty units / CTAs)
// non-empty units (tickets are claimed one unit ahead; without the quota a CTA
// whose first units were cheap would take one more than the rest), and chunks
// wholly past their row's length are zeroed by a static share per CTA.
//
// Chunk-local frames. Each unit rotates q and k by the phase accumulated from
// its own chunk start, so its scores and its state contribution
//   dS_c^T = kr_c^T (v_c * scale * 2^(total_c - cs))              (n x p)
// need nothing from earlier chunks. Because q and k of a pair rotate by the
// same angle, the state entering chunk c, in chunk c's frame, is
//   S(0) = 0,   S(x+1) = R(-theta_x) (2^total_x S(x) + dS_x),
// with theta_x chunk x's summed angle increment and R the rotation of the
// first 32 (even, odd) pairs of the state's n axis. In real arithmetic this is
// the reference's serial recurrence (mamba_fused.py:93-152).
//
// Exchange through L2. After its first MMAs a unit publishes dS_c (FP16 with a
// power-of-two exponent per half row), theta_c and 2^total_c in the workspace
// and raises its flag. A later unit folds its predecessors' contributions.
// For long rows (more than 8 chunks) every unit also publishes its outgoing
// state S(c+1) (FP32) once known, and a successor looks back only to the
// nearest predecessor whose outgoing state is available (decoupled look-back).
// Flags carry a launch epoch, so the workspace needs no clearing between
// launches; the last CTA to finish advances the epoch and resets the ticket.
//
// Roles inside a CTA (512 threads, one CTA per SM, two pipeline slots):
//   warps 0-7   producer: controls, phases, FP16 operand tiles from the rows
//               staged in shared memory by cp.async during the previous unit;
//               stages the next unit's rows; warp 7 claims its ticket, warp 6
//               issues this unit's scores / state MMAs (MMA 1) after the next
//               iteration's first barriers;
//   warps 8-15  epilogue (two warps per TMEM lane quarter, one per 32-column
//               half): export dS, decayed scores -> P tiles, MMA 2 (P v),
//               fold -> S tile, MMA 3 (q S^T), gated output, release the slot.
//
// Tensor-core work per unit (tcgen05.mma kind::f16, FP16 operands in
// 128B-swizzled shared memory, FP32 accumulators in tensor memory):
//   scores  D_s  = q16 k16^T              M=64  N=64 K=128
//   state   D_d  = k16^T (vs_hi + vs_lo)  M=128 N=64 K=64 x2  (k16 read MN-major)
//   values  D_pv = (P_hi + P_lo) v16      M=64  N=64 K=64 x2
//   inter   D_i  = q16 S^T                M=64  N=64 K=128
// Precision: FP16 operands carry per-row power-of-two exponents (undone exactly
// after the MMA); the decayed scores P and the decay-weighted values vs are
// split into FP16 hi + lo halves; sums accumulate in FP32. qk (the D-skip dot
// product, mamba_fused.py:124) is the score diagonal, since rotating q and k by
// the same angle preserves their dot product; (D + qk) v rides on P's diagonal.
#include <cstdio>
#include <initializer_list>

#include "../../include/trifusion_b200.h"
#include <cudaTypedefs.h>

#include "recurrence.cuh"
#include "sm100.cuh"
#include "tf_host.cuh"

namespace tf {
namespace {

using namespace sm100;

constexpr int kThreads = 512;
constexpr int kProducerThreads = 256;  // warps 0-7
constexpr int kEpilogueThreads = 256;  // warps 8-15
constexpr int kBarProducer = 1, kBarEpilogue = 2, kBarPair = 3;  // kBarPair + quarter: 3..6
constexpr int kClaimThread = 224;      // producer thread that claims the next unit's ticket
constexpr int kMmaThread = 192;        // producer thread that issues MMA 1
constexpr int kLookbackChunks = 8;     // rows with more chunks publish outgoing states

// ---- shared memory --------------------------------------------------------------
// Per slot (bytes from the slot base, 1024-aligned). The k and vs tiles are read
// only by MMA 1; the epilogue starts after MMA 1 has completed, so its P hi/lo
// tiles reuse the k tile. The S^T tile reuses the vs and v16 tiles once MMA 2
// (the last reader of v16) has completed.
constexpr uint32_t kSlotQ = 0;        // q16  K-major  [2 K-blocks][64 rows][128 B]
constexpr uint32_t kSlotK = 16384;    // k~   K-major  [2 K-blocks][64 rows][128 B]
constexpr uint32_t kSlotPH = 16384;   // P hi K-major [64 rows][128 B]   (over k~, after MMA 1)
constexpr uint32_t kSlotPL = 24576;   // P lo                            (over k~, after MMA 1)
constexpr uint32_t kSlotVS = 32768;   // vs   MN-major [64 rows][128 B]
constexpr uint32_t kSlotV = 40960;    // v16  MN-major [64 rows][128 B]
constexpr uint32_t kSlotS = 32768;    // S^T MN-major [128 rows][128 B]  (over vs and v16, after MMA 2)
constexpr uint32_t kSlotZ = 49152;    // z in / out staging, BF16 [64 rows][128 B]
constexpr uint32_t kSlotBytes = 57344;
// Staging of the next unit's raw rows, filled by cp.async while the current unit
// is prepared. Each producer thread copies and later reads back only its own
// 16-byte chunks ([chunk][thread] order: a warp's accesses are contiguous); the
// angle rows ([64][32] BF16) are read across threads after a barrier.
constexpr uint32_t kOffStage = 2 * kSlotBytes;
constexpr uint32_t kStQ = 0, kStK = 16384, kStV = 32768, kStZ = 40960, kStA = 49152, kStageBytes = 53248;
// With TMA staging the same regions hold boxes of 64 time steps in time order:
// q and k as two [64][128 B] 128B-swizzled boxes (columns 0-63, 64-127), v and z as
// one each, the angles as [64][64 B]; all 53248 bytes arrive on one mbarrier.
constexpr uint32_t kStageTmaBytes = 53248;
// Producer scratch and barriers after the staging area.
constexpr uint32_t kOffPhase = kOffStage + kStageBytes;  // FP32 [64][33]
constexpr uint32_t kOffTeff = kOffPhase + 64 * 33 * 4;   // int [2][kTeffTable]: valid length of every row
constexpr int kTeffTable = 1024;                          // batches beyond this read lengths[] directly
// Ticket map (launches of at most kMapRows rows and kMapChunks chunks per row): the rows
// ordered by valid length, longest first (short), and per chunk c the number of
// non-empty units of the chunks before c (int, kMapChunks + 1 entries).
constexpr int kMapRows = 256, kMapChunks = 512;
constexpr uint32_t kOffMap = kOffTeff + 2 * kTeffTable * 4;
constexpr uint32_t kOffMisc = kOffMap + ((kMapRows * 2 + (kMapChunks + 1) * 4 + 15) & ~15u);

struct SlotHeader {
  int unit;  // -1: no more work
  int b, h, c, nv;
  int dir, teff;        // direction of the unit, valid length of its row
  float cs[kChunk];     // decay cumsum (log2 units)
  float g[kChunk];      // gamma_i / scale_i (0 where scale_i is 0): the D-skip term on P's diagonal
  float qe[kChunk];     // q16 row exponents
  float rl[kChunk];     // log2 of P's row factor: cs_i - mu - qe_i
  float cl[kChunk];     // log2 of P's column factor: n_j - ke_j (an integer)
  float cf[kChunk];     // 2^cl_j (units that are not wide)
  float pe[kChunk];     // P row exponents (epilogue)
  float pmax[2][kChunk];  // per column half (epilogue)
  float theta[kRotary];
  float gtot;
  float sinv;           // 2^-(state tile exponent) (epilogue)
  int wide;             // decay range over 180 binades: P's factors are combined per element
};
struct Misc {
  SlotHeader hdr[2];
  float scale[kChunk];  // producer scratch
  float dtc[kChunk];
  float seg[8][kRotary];
  float wsum[2];
  float csmax[2], csmin[2];  // decay cumsum range (warps 0-1)
  float ered[8];        // epilogue reductions
  int ticket;
  int next_ticket;
  int lookback_start;
  int quota;            // non-empty units one CTA takes at most
  uint32_t epoch;
  uint32_t tmem_base;
  uint64_t ready[2], freed[2], mma1[2], mma2[2], mma3[2];
  uint64_t staged;  // TMA staging of the next unit's rows
};
constexpr uint32_t kSmemBytes = kOffMisc + sizeof(Misc) + 1024;
static_assert(kSmemBytes <= 232448, "shared memory beyond the 227 KB a B200 CTA may use");

constexpr uint32_t kColS = 0, kColD = 64, kColPV = 128, kColI = 192, kSlotCols = 256, kTmemCols = 512;

constexpr uint32_t kIdScore = idesc_f16_f32(64, 64, false, false);
constexpr uint32_t kIdState = idesc_f16_f32(128, 64, true, true);
constexpr uint32_t kIdPV = idesc_f16_f32(64, 64, false, true);
constexpr uint32_t kIdInter = idesc_f16_f32(64, 64, false, true);

// ---- workspace ------------------------------------------------------------------
// [header: epoch | ticket | done, each on its own 128-byte line]
// per unit: [flag (128 B line)] [theta 32 + gtot (256 B)] [half-row exponent
// factors 2x128 FP32 (1 KB)] [dS^T FP16 128x64 (16 KB)] [S(c+1)^T FP32 128x64 (32 KB)]
constexpr size_t kWsHeader = 384;
constexpr size_t kUnitFlag = 0, kUnitTheta = 128, kUnitExp = 384, kUnitAgg = 1408, kUnitIncl = 1408 + 16384;
constexpr size_t kUnitBytes = kUnitIncl + 32768;
constexpr uint32_t kFlagAgg = 1, kFlagIncl = 2, kEpochStep = 2;

// ---- helpers --------------------------------------------------------------------
template <int kVec>
__device__ __forceinline__ uint4 load16(const bf16* p) {
  if constexpr (kVec == 16) {
    return __ldg(reinterpret_cast<const uint4*>(p));
  } else if constexpr (kVec == 8) {
    const uint2 a = __ldg(reinterpret_cast<const uint2*>(p));
    const uint2 b = __ldg(reinterpret_cast<const uint2*>(p + 4));
    return make_uint4(a.x, a.y, b.x, b.y);
  } else {
    const unsigned short* s = reinterpret_cast<const unsigned short*>(p);
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) w[i] = static_cast<uint32_t>(s[2 * i]) | (static_cast<uint32_t>(s[2 * i + 1]) << 16);
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
}
template <int kVec>
__device__ __forceinline__ void store16(bf16* p, uint4 v) {
  if constexpr (kVec == 16) {
    *reinterpret_cast<uint4*>(p) = v;
  } else if constexpr (kVec == 8) {
    *reinterpret_cast<uint2*>(p) = make_uint2(v.x, v.y);
    *reinterpret_cast<uint2*>(p + 4) = make_uint2(v.z, v.w);
  } else {
    unsigned short* s = reinterpret_cast<unsigned short*>(p);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      s[2 * i] = static_cast<unsigned short>(w[i] & 0xffffu);
      s[2 * i + 1] = static_cast<unsigned short>(w[i] >> 16);
    }
  }
}
__device__ __forceinline__ void unpack8(uint4 u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(w[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t a) {
  asm volatile("st.shared.b32 [%0], %1;" ::"r"(addr), "r"(a) : "memory");
}
__device__ __forceinline__ uint32_t ld_shared_u32(uint32_t addr) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}
__device__ __forceinline__ uint32_t ld_shared_u16(uint32_t addr) {
  unsigned short v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(addr));
  return v;
}
// Asynchronous global -> shared copies (zero-filled beyond `src_bytes`; a
// zero-byte copy reads nothing and writes zeros).
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async8(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// 16 bytes of a row (16- or 8-byte aligned) into shared memory, or zeros.
template <int kVec>
__device__ __forceinline__ void stage16(uint32_t dst, const bf16* src, bool valid) {
  if constexpr (kVec == 16) {
    cp_async16(dst, src, valid ? 16u : 0u);
  } else {
    cp_async8(dst, src, valid ? 8u : 0u);
    cp_async8(dst + 8, src + 4, valid ? 8u : 0u);
  }
}
__device__ __forceinline__ uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}
// 16 TMEM lanes x 32 columns in the m16n8 fragment order: thread t gets lanes
// t/4 and t/4+8, columns 8k + 2(t%4) + {0,1} (k = 0..3) as r[4k+0..1] (lane
// t/4) and r[4k+2..3] (lane t/4+8).
__device__ __forceinline__ void tmem_ld_16x256_x4(uint32_t taddr, float (&r)[16]) {
  uint32_t* u = reinterpret_cast<uint32_t*>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.16x256b.x4.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
        "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void bar_sync_n(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int atom_add_acq_rel(int* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ uint4 ld_cg_v4(const void* p) {
  return __ldcg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ float load_trap(const RecurrenceParams& p, const char* base, int64_t off) {
  return p.trap_bf16 ? bf2f(reinterpret_cast<const bf16*>(base)[off]) : reinterpret_cast<const float*>(base)[off];
}
__device__ __forceinline__ int ilog2_or(float max_abs, int if_zero) {
  if (!(max_abs > 0.f)) return if_zero;
  return static_cast<int>((__float_as_uint(max_abs) >> 23) & 0xffu) - 127;
}
__device__ __forceinline__ float silu_tanh(float z) {
  const float hz = 0.5f * z;
  return fmaf(hz, tanh_approx(hz), hz);  // z * sigmoid(z) = hz (1 + tanh(hz))
}

__device__ int g_device_error = 0;  // 1: a bounded wait gave up; 2: an out-of-range access (bounds build)

// [off, off + width) within a tensor of `ext` elements. Always true, except in a
// build with TF_DEBUG_BOUNDS, where a range outside records error 2 and returns
// false: the caller then reads zeros (or element 0) or skips the store.
// An offset to use only when `ok` (bounds build: element 0 otherwise; other builds
// use the offset as it is, where `ok` is always the caller's own row validity).
#ifdef TF_DEBUG_BOUNDS
#define TF_OFF(ok, off) ((ok) ? (off) : 0)
#else
#define TF_OFF(ok, off) (off)
#endif
__device__ __forceinline__ bool tf_in(int64_t off, int64_t width, int64_t ext) {
#ifdef TF_DEBUG_BOUNDS
  if (off >= 0 && off + width <= ext) return true;
  atomicExch(&g_device_error, 2);
  return false;
#else
  (void)off, (void)width, (void)ext;
  return true;
#endif
}

__device__ __forceinline__ float2 pair(const float* x) { return make_float2(x[0], x[1]); }
__device__ __forceinline__ void set_pair(float* x, float2 v) {
  x[0] = v.x;
  x[1] = v.y;
}
// One producer thread's 32 elements of a q or k row (8-element vectors i = 0..3
// at columns 32 i + 8 s4): optional RMSNorm with FP32 statistics (weights w),
// (output rounded to BF16, the reference's tensor type), bias, and the rotation
// of the two vectors that hold rotating pairs. Returns
// the row's max |x| over its four threads. Paired FP32 arithmetic (exact per
// lane) halves the instruction count. Rows past the valid length are left as
// computed: their outputs are never stored and their decay-weighted values are
// zero, so they contribute nothing.
__device__ __forceinline__ float prep_qk_row(float (&x)[32], const uint4 (&raw)[4], const float* __restrict__ w,
                                             float eps, const float* __restrict__ bias, int s4,
                                             const float (&cn)[8], const float (&sn)[8]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) unpack8(raw[i], &x[8 * i]);
  if (w) {  // RMSNorm (native.py:8-39)
    float2 acc = make_float2(0.f, 0.f);
#pragma unroll
    for (int m = 0; m < 16; ++m) acc = __ffma2_rn(pair(&x[2 * m]), pair(&x[2 * m]), acc);
    float ss = acc.x + acc.y;
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    const float rr = rsqrtf(ss * (1.f / kState) + eps);
    const float2 r2 = make_float2(rr, rr);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float4 w0 = __ldg(reinterpret_cast<const float4*>(w + 32 * i + 8 * s4));
      const float4 w1 = __ldg(reinterpret_cast<const float4*>(w + 32 * i + 8 * s4 + 4));
      const float2 wp[4] = {make_float2(w0.x, w0.y), make_float2(w0.z, w0.w), make_float2(w1.x, w1.y),
                            make_float2(w1.z, w1.w)};
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        // The norm's output is a BF16 tensor in the reference (native.py:37-38): round it.
        const float2 y = __fmul2_rn(__fmul2_rn(pair(&x[8 * i + 2 * m]), r2), wp[m]);
        set_pair(&x[8 * i + 2 * m], __bfloat1622float2(__float22bfloat162_rn(y)));
      }
    }
  }
  float mx = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4 b0 = __ldg(reinterpret_cast<const float4*>(bias + 32 * i + 8 * s4));
    const float4 b1 = __ldg(reinterpret_cast<const float4*>(bias + 32 * i + 8 * s4 + 4));
    const float2 bp[4] = {make_float2(b0.x, b0.y), make_float2(b0.z, b0.w), make_float2(b1.x, b1.y),
                          make_float2(b1.z, b1.w)};
#pragma unroll
    for (int m = 0; m < 4; ++m) set_pair(&x[8 * i + 2 * m], __fadd2_rn(pair(&x[8 * i + 2 * m]), bp[m]));
    if (i < 2) {
#pragma unroll
      for (int m = 0; m < 4; ++m) {
        // (a0 c - a1 s, a0 s + a1 c) = (a0, a0) * (c, s) + (a1, a1) * (-s, c)
        const float a0 = x[8 * i + 2 * m], a1 = x[8 * i + 2 * m + 1];
        const float c = cn[4 * i + m], sv = sn[4 * i + m];
        const float2 tt = __fmul2_rn(make_float2(a1, a1), make_float2(-sv, c));
        set_pair(&x[8 * i + 2 * m], __ffma2_rn(make_float2(a0, a0), make_float2(c, sv), tt));
      }
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) mx = fmaxf(mx, fabsf(x[8 * i + e]));
  }
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
  mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
  return mx;
}

struct Shape {
  int B, H, nck, units, ndir;
};
// Units are numbered chunk-major, then direction: u = ((c*ndir + dir)*B + b)*H + h.
__device__ __forceinline__ void decode_unit(int u, const Shape& s, int& b, int& h, int& c, int& dir) {
  h = u % s.H;
  int rest = u / s.H;
  b = rest % s.B;
  rest /= s.B;
  dir = rest % s.ndir;
  c = rest / s.ndir;
}
__device__ __forceinline__ int unit_index(const Shape& s, int c, int dir, int b, int h) {
  return ((c * s.ndir + dir) * s.B + b) * s.H + h;
}
// The controls of mamba.py:58-63 / kernels/primitives.py:190-216, in the same
// FP32 operations as the standalone controls kernel.
__device__ __forceinline__ float softplus_dt(float v) { return v > 20.f ? v : log1pf(expf(v)); }
__device__ __forceinline__ float a_control(float a, float floor_) {
  return fminf(-(fmaxf(a, 0.f) + 1.f / (1.f - fminf(a, 0.f))), -floor_);
}
__device__ __forceinline__ unsigned char* unit_ws(unsigned char* ws, int u) {
  return ws + kWsHeader + static_cast<size_t>(u) * kUnitBytes;
}
// Spin (bounded in time) until a unit's flag reaches `want` in this launch's epoch.
// `limit_ns` is the launch's flag-wait limit (2 s unless the caller lowered it).
__device__ __forceinline__ bool wait_flag(const uint32_t* flag, uint32_t epoch, uint32_t want, uint32_t& seen,
                                          uint64_t limit_ns) {
  seen = ld_acquire_u32(flag);
  if (static_cast<int>(seen - epoch) >= static_cast<int>(want)) return true;
  const uint64_t t0 = global_timer_ns();
  for (;;) {
    __nanosleep(64);
    seen = ld_acquire_u32(flag);
    if (static_cast<int>(seen - epoch) >= static_cast<int>(want)) return true;
    if (global_timer_ns() - t0 > limit_ns) return false;
  }
}

// =====================================================================================
// kDirs: directions in the launch (1 or 2), a compile-time constant so that a
// one-direction launch reads its parameters at fixed offsets. kExt: reversed
// rows and in-launch controls are possible (otherwise compiled out).
// kTma: the unit's rows are staged by TMA boxes (16-byte rows whose tensor maps the
// launcher could encode); otherwise by per-thread cp.async (or read directly).
template <int kVec, int kDirs, bool kExt, bool kLook, bool kTma>
__device__ __forceinline__ void recurrence_body(const RecurrenceParams& pd0, const RecurrenceParams& pd1,
                                                unsigned char* ws) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  unsigned char* smem = smem_raw + (base - raw_addr);
  Misc& mi = *reinterpret_cast<Misc*>(smem + kOffMisc);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  uint32_t* ws_epoch = reinterpret_cast<uint32_t*>(ws);
  int* ws_ticket = reinterpret_cast<int*>(ws + 128);
  int* ws_done = reinterpret_cast<int*>(ws + 256);
  const RecurrenceParams& p0 = pd0;
  const int nck = (p0.T + kChunk - 1) / kChunk;
  const Shape shp{p0.B, p0.H, nck, nck * kDirs * p0.B * p0.H, kDirs};
  // A unit's workspace record (unit 0's, with error 2 recorded, if u is out of range).
  auto uws_of = [&](int u) { return unit_ws(ws, TF_OFF(tf_in(u, 1, shp.units), u)); };
  constexpr bool lookback = kLook;  // rows longer than kLookbackChunks chunks (chosen by the launcher)
  // Valid length of every row (per direction), read once per CTA.
  int* teff_tab = reinterpret_cast<int*>(smem + kOffTeff);
  auto row_length = [&](const RecurrenceParams& pr, int bb) -> int {
    if (!pr.lengths) return pr.T;
    const int64_t len = tf_in(bb, 1, pr.B) ? pr.lengths[bb] : 0;
    return static_cast<int>(len < 0 ? 0 : (len > pr.T ? pr.T : len));
  };
  if (p0.B <= kTeffTable) {
    for (int i = tid; i < kDirs * p0.B; i += kThreads) {
      const int dd = i / p0.B;
      teff_tab[dd * kTeffTable + (i - dd * p0.B)] = row_length(dd == 0 ? pd0 : pd1, i - dd * p0.B);
    }
  }
  auto teff_of = [&](int dd, int bb, const RecurrenceParams& pr) -> int {
    return p0.B <= kTeffTable ? teff_tab[dd * kTeffTable + bb] : row_length(pr, bb);
  };

  // ---- ticket map: tickets -> non-empty units -------------------------------------
  // Built by warps 1-15 while warp 0 allocates TMEM and sets up the barriers.
  const bool use_map = p0.B <= kTeffTable && kDirs * p0.B <= kMapRows && nck <= kMapChunks;
  short* map_order = reinterpret_cast<short*>(smem + kOffMap);
  int* map_pref = reinterpret_cast<int*>(smem + kOffMap + kMapRows * 2);
  if (use_map) {
    __syncthreads();  // the length table is complete
    if (warp > 0) {
      const int nrows = kDirs * p0.B;
      auto teff_row = [&](int i) { return i < p0.B ? teff_tab[i] : teff_tab[kTeffTable + i - p0.B]; };
      for (int i = tid - 32; i < nrows; i += kThreads - 32) {  // rank of row i: longer rows first, ties by index
        const int ti = teff_row(i);
        int rank = 0;
        for (int j = 0; j < nrows; ++j) {
          const int tj = teff_row(j);
          rank += (tj > ti) | ((tj == ti) & (j < i));
        }
        map_order[rank] = static_cast<short>(i);
      }
      for (int c = tid - 32; c <= nck; c += kThreads - 32) {  // non-empty units of the chunks before c
        int before = 0;
        for (int j = 0; j < nrows; ++j) before += min((teff_row(j) + kChunk - 1) / kChunk, c);
        map_pref[c] = before * p0.H;
      }
    }
  }

  if (warp == 0) {
    tmem_alloc(&mi.tmem_base, kTmemCols);
    tmem_relinquish();
  }
  if (kTma && tid == kClaimThread) {
#pragma unroll
    for (int d = 0; d < kDirs; ++d) {
      const RecurrenceParams& pp = d == 0 ? pd0 : pd1;
      prefetch_tensormap(&pp.tm_q);
      prefetch_tensormap(&pp.tm_k);
      prefetch_tensormap(&pp.tm_v);
      prefetch_tensormap(&pp.tm_z);
      prefetch_tensormap(&pp.tm_a);
    }
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&mi.ready[s], 1);
      mbar_init(&mi.freed[s], 1);
      mbar_init(&mi.mma1[s], 1);
      mbar_init(&mi.mma2[s], 1);
      mbar_init(&mi.mma3[s], 1);
    }
    mbar_init(&mi.staged, 1);
    fence_mbar_init();
    // The first unit's ticket, claimed now so its round trip overlaps the epoch
    // and length loads (the previous launch reset the counter before it ended).
    const int first = atomicAdd(ws_ticket, 1);
    mi.epoch = ld_acquire_u32(ws_epoch);
    mi.next_ticket = first;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem0 = mi.tmem_base;
  const uint32_t epoch = mi.epoch;
  bool ok = true;

  // The unit of ticket tk (shp.units once every non-empty unit is handed out).
  auto ticket_unit = [&](int tk) -> int {
    if (!use_map) return tk;
    if (tk >= map_pref[nck]) return shp.units;
    int lo = 0, hi = nck;  // map_pref[lo] <= tk < map_pref[hi]
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (map_pref[mid] <= tk) lo = mid; else hi = mid;
    }
    const int r = tk - map_pref[lo];
    const int row = map_order[r / p0.H];
    const int dd = row >= p0.B ? 1 : 0;
    return unit_index(shp, lo, dd, row - dd * p0.B, r % p0.H);
  };

  if (warp < 8) {
    // =========================== producer ===========================
    const int t = tid >> 2, s4 = tid & 3;  // row, sub-slot (4 threads per row)
    int k = 0;                             // slot uses so far
    constexpr bool kStage = kVec >= 8;     // rows aligned for 8/16-byte cp.async
    const uint32_t stage = base + kOffStage;
    // Stage unit un's q/k/v/z rows (this thread's chunks) and angle rows.
    bool tma_pending = false;  // TMA boxes of a staged unit in flight on mi.staged
    uint32_t tma_phase = 0;
    auto stage_unit = [&](int un) {
      if constexpr (kStage) {
        if (un >= shp.units) return;
        int nb, nh, nc, nd;
        decode_unit(un, shp, nb, nh, nc, nd);
        if (kDirs == 1) nd = 0;
        const RecurrenceParams& pn = (kDirs == 1 || nd == 0) ? pd0 : pd1;
        const int te = teff_of(nd, nb, pn);
        const int nvn = max(0, min(kChunk, te - nc * kChunk));
        if (nvn == 0) return;
        const bool rv = kExt && pn.reverse != 0;
        if constexpr (kTma) {
          // One thread issues the unit's boxes: 64 time steps starting at the chunk's
          // first step, or (reversed rows) at len - 64 - c0, read in reverse below.
          // Steps before 0 or past T read as zeros.
          if (tid == kClaimThread) {
            const int row0 = rv ? te - kChunk - nc * kChunk : nc * kChunk;
            const int hq = nh / (pn.H / pn.Hq);
            fence_async_smem();  // the previous unit's rows were read through the generic proxy
            mbar_arrive_expect_tx(&mi.staged, kStageTmaBytes);
            tma_load_4d(stage + kStQ, &pn.tm_q, &mi.staged, 0, hq, row0, nb);
            tma_load_4d(stage + kStQ + 8192u, &pn.tm_q, &mi.staged, 64, hq, row0, nb);
            tma_load_4d(stage + kStK, &pn.tm_k, &mi.staged, 0, hq, row0, nb);
            tma_load_4d(stage + kStK + 8192u, &pn.tm_k, &mi.staged, 64, hq, row0, nb);
            tma_load_4d(stage + kStV, &pn.tm_v, &mi.staged, 0, nh, row0, nb);
            tma_load_4d(stage + kStZ, &pn.tm_z, &mi.staged, 0, nh, row0, nb);
            tma_load_4d(stage + kStA, &pn.tm_a, &mi.staged, 0, pn.sa[2] == 0 ? 0 : nh, row0, nb);
          }
          tma_pending = true;
          return;
        }
        const bool valid = t < nvn;
        const int64_t x = static_cast<int64_t>(nc) * kChunk + t;
        const int64_t pos = valid ? (rv ? te - 1 - x : x) : 0;
        const int hq = nh / (pn.H / pn.Hq);
        const int64_t qo = nb * pn.sq[0] + pos * pn.sq[1] + hq * pn.sq[2];
        const int64_t ko = nb * pn.sk[0] + pos * pn.sk[1] + hq * pn.sk[2];
        const int64_t vo = nb * pn.sv[0] + pos * pn.sv[1] + nh * pn.sv[2];
        const int64_t zo = nb * pn.sz[0] + pos * pn.sz[1] + nh * pn.sz[2];
        const bool qv = valid && tf_in(qo, kState, pn.ext_q), kv = valid && tf_in(ko, kState, pn.ext_k);
        const bool vv = valid && tf_in(vo, kHead, pn.ext_v), zv = valid && tf_in(zo, kHead, pn.ext_z);
        const bf16* qrow = pn.q + TF_OFF(qv, qo);
        const bf16* krow = pn.k + TF_OFF(kv, ko);
        const bf16* vrow = pn.v + TF_OFF(vv, vo);
        const bf16* zrow = pn.z + TF_OFF(zv, zo);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          stage16<kVec>(stage + kStQ + i * 4096u + tid * 16u, qrow + 32 * i + 8 * s4, qv);
          stage16<kVec>(stage + kStK + i * 4096u + tid * 16u, krow + 32 * i + 8 * s4, kv);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          stage16<kVec>(stage + kStV + i * 4096u + tid * 16u, vrow + 32 * i + 8 * s4, vv);
          stage16<kVec>(stage + kStZ + i * 4096u + tid * 16u, zrow + 32 * i + 8 * s4, zv);
        }
        if (pn.ang_vec) {  // row tid/4, pairs 8*(tid%4) .. +7
          const int ra = tid >> 2;
          const int64_t xa = static_cast<int64_t>(nc) * kChunk + ra;
          const int64_t apos = ra < nvn ? (rv ? te - 1 - xa : xa) : 0;
          const int64_t ao = nb * pn.sa[0] + apos * pn.sa[1] + nh * pn.sa[2] + 8 * s4;
          const bool av = ra < nvn && tf_in(ao, 8, pn.ext_a);
          const bf16* arow = pn.ang + TF_OFF(av, ao);
          cp_async8(stage + kStA + ra * 64u + s4 * 16u, arow, av ? 8u : 0u);
          cp_async8(stage + kStA + ra * 64u + s4 * 16u + 8u, arow + 4, av ? 8u : 0u);
        }
        cp_async_commit();
      }
    };
    // MMA 1 (scores and state) of a finished slot. One thread of warp 6 issues it
    // after the next iteration's first barriers, so the other 255 threads do not
    // wait for the issue; warp 6 has slack there (warps 0-1 load the controls).
    int pend = -1;
    auto issue_mma1 = [&](int s) {
      tc_fence_after();
      const uint32_t sbs = base + s * kSlotBytes;
      const uint32_t tm = tmem0 + s * kSlotCols;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t koff = (kk >> 2) * 8192u + (kk & 3) * 32u;
        umma_f16(tm + kColS, desc_sw128(sbs + kSlotQ + koff, 0, 1024), desc_sw128(sbs + kSlotK + koff, 0, 1024),
                 kIdScore, kk > 0);
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk)
        umma_f16(tm + kColD, desc_sw128(sbs + kSlotK + kk * 2048u, 8192, 1024),
                 desc_sw128(sbs + kSlotVS + kk * 2048u, 8192, 1024), kIdState, kk > 0);
      umma_commit(&mi.mma1[s]);
      mbar_arrive(&mi.ready[s]);
    };
    // Quota: ceil(non-empty units / CTAs). Tickets are claimed one unit ahead, so
    // without it a CTA whose first units were cheap runs one unit more than the
    // rest and sets the launch's end. A CTA at its quota stops claiming; the
    // others, below it, claim what is left (CTAs x quota >= non-empty units).
    if (warp == 0) {
      long long nonempty = 0;
      if (p0.B <= kTeffTable) {
        for (int i = lane; i < kDirs * p0.B; i += 32) nonempty += (teff_tab[(i / p0.B) * kTeffTable + i % p0.B] + kChunk - 1) / kChunk;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) nonempty += __shfl_xor_sync(0xffffffffu, nonempty, o);
        nonempty *= p0.H;
      }
      if (lane == 0) {
        const long long g = gridDim.x;
        mi.quota = p0.B <= kTeffTable ? static_cast<int>((nonempty + g - 1) / g) : 0x7fffffff;
        mi.next_ticket = ticket_unit(mi.next_ticket);  // the first ticket, claimed at set-up
      }
    }
    bar_sync_n(kBarProducer, kProducerThreads);
    const int quota = mi.quota;
    int held = 0;  // non-empty units this CTA has taken
    stage_unit(mi.next_ticket);
    for (;;) {
      if constexpr (kStage) cp_async_wait_all();
      if constexpr (kTma) {
        if (tma_pending) {
          ok &= mbar_spin(&mi.staged, tma_phase);
          tma_phase ^= 1u;
          tma_pending = false;
        }
      }
      bar_sync_n(kBarProducer, kProducerThreads);  // staged rows and the ticket are visible
      const int u = mi.next_ticket;
      bar_sync_n(kBarProducer, kProducerThreads);  // everyone has read the ticket
      if (pend >= 0) {
        if (tid == kMmaThread) issue_mma1(pend);
        pend = -1;
      }
      int my_next = shp.units;  // no further unit unless claimed below
      const int slot = k & 1;
      SlotHeader& hd = mi.hdr[slot];
      if (u >= shp.units) {
        // Tell the epilogue there is no more work, through the next slot.
        if (k >= 2) ok &= mbar_wait(&mi.freed[slot], ((k >> 1) - 1) & 1);
        if (tid == 0) {
          hd.unit = -1;
          mbar_arrive(&mi.ready[slot]);
        }
        break;
      }
      int b, h, c, dir;
      decode_unit(u, shp, b, h, c, dir);
      if (kDirs == 1) dir = 0;
      const RecurrenceParams& p = (kDirs == 1 || dir == 0) ? pd0 : pd1;
      const int T_eff = teff_of(dir, b, p);
      const int c0 = c * kChunk;
      const int nv = max(0, min(kChunk, T_eff - c0));
      // Request the following unit now (below the quota); the atomic stays in
      // flight while this unit's loads complete, and its rows are staged once
      // the controls are done.
      held += nv > 0;
      // (Claimed by warp 7, which has less other single-thread work than warp 0.)
      // Short rows claim at once; long rows once the unit's tiles are under way (below):
      // the later a unit is claimed, the fewer of its row's predecessors are still
      // unpublished when its epilogue looks back.
      if (!kLook && tid == kClaimThread && held < quota) my_next = ticket_unit(atomicAdd(ws_ticket, 1));
      if (nv == 0) {
        // Whole chunk past the length: no tensor work, no slot; its rows are
        // zeroed after the loop. (Every later chunk of this row is empty too,
        // so nobody reads its state.)
        if (kLook && tid == kClaimThread && held < quota) my_next = ticket_unit(atomicAdd(ws_ticket, 1));
        if (tid == kClaimThread) mi.next_ticket = my_next;
        bar_sync_n(kBarProducer, kProducerThreads);
        stage_unit(mi.next_ticket);
        continue;
      }
      const bool row_ok = t < nv;
      // Time of local step x of this row: x itself, or len-1-x for a reversed row.
      const bool rev = kExt && p.reverse != 0;
      auto src_row = [&](int64_t x) -> int64_t { return rev ? (T_eff - 1 - x) : x; };
      // ---- loads ------------------------------------------------------------------
      uint4 qraw[4], kraw[4], vraw[2], zraw[2];
      constexpr bool tma_rows = kTma;
      if constexpr (tma_rows) {
        // Boxes in time order: local step t is box row t, or 63 - t for reversed rows.
        const int r = rev ? kChunk - 1 - t : t;
        const uint32_t off0 = r * 128u + (((s4 ^ r) & 7u) << 4), off1 = r * 128u + ((((4 + s4) ^ r) & 7u) << 4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const uint32_t off = (i >> 1) * 8192u + ((i & 1) ? off1 : off0);
          qraw[i] = ld_shared_v4(stage + kStQ + off);
          kraw[i] = ld_shared_v4(stage + kStK + off);
        }
        vraw[0] = ld_shared_v4(stage + kStV + off0);
        vraw[1] = ld_shared_v4(stage + kStV + off1);
        zraw[0] = ld_shared_v4(stage + kStZ + off0);
        zraw[1] = ld_shared_v4(stage + kStZ + off1);
        if (nv < kChunk && !row_ok) {
          // A row's last chunk: the boxes hold whatever lies past the length; use zeros
          // (as the reference's masked loads do).
          const uint4 zero = make_uint4(0, 0, 0, 0);
#pragma unroll
          for (int i = 0; i < 4; ++i) qraw[i] = kraw[i] = zero;
          vraw[0] = vraw[1] = zraw[0] = zraw[1] = zero;
        }
      } else if constexpr (kStage) {
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          qraw[i] = ld_shared_v4(stage + kStQ + i * 4096u + tid * 16u);
          kraw[i] = ld_shared_v4(stage + kStK + i * 4096u + tid * 16u);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          vraw[i] = ld_shared_v4(stage + kStV + i * 4096u + tid * 16u);
          zraw[i] = ld_shared_v4(stage + kStZ + i * 4096u + tid * 16u);
        }
      } else {
        const int64_t pos = row_ok ? src_row(c0 + t) : 0;
        const int64_t qo = b * p.sq[0] + pos * p.sq[1] + (h / (p.H / p.Hq)) * p.sq[2];
        const int64_t ko = b * p.sk[0] + pos * p.sk[1] + (h / (p.H / p.Hq)) * p.sk[2];
        const int64_t vo = b * p.sv[0] + pos * p.sv[1] + h * p.sv[2];
        const int64_t zo = b * p.sz[0] + pos * p.sz[1] + h * p.sz[2];
        const bool qv = row_ok && tf_in(qo, kState, p.ext_q), kv = row_ok && tf_in(ko, kState, p.ext_k);
        const bool vv = row_ok && tf_in(vo, kHead, p.ext_v), zv = row_ok && tf_in(zo, kHead, p.ext_z);
        const bf16* qrow = p.q + TF_OFF(qv, qo);
        const bf16* krow = p.k + TF_OFF(kv, ko);
        const bf16* vrow = p.v + TF_OFF(vv, vo);
        const bf16* zrow = p.z + TF_OFF(zv, zo);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int e = 32 * i + 8 * s4;
          qraw[i] = qv ? load16<kVec>(qrow + e) : make_uint4(0, 0, 0, 0);
          kraw[i] = kv ? load16<kVec>(krow + e) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
          const int e = 32 * i + 8 * s4;
          vraw[i] = vv ? load16<kVec>(vrow + e) : make_uint4(0, 0, 0, 0);
          zraw[i] = zv ? load16<kVec>(zrow + e) : make_uint4(0, 0, 0, 0);
        }
      }
      float c_dt = 0.f, c_dn = 0.f, c_tr = 0.f, c_tn = 0.f, c_adt = 0.f;
      if (tid < kChunk) {
        const float* dtbase = p.dt + b * p.sdt[0] + h * p.sdt[1];
        const float* adtbase = p.adt + b * p.sadt[0] + h * p.sadt[1];
        const char* trbase =
            static_cast<const char*>(p.trap) + (b * p.str[0] + h * p.str[1]) * (p.trap_bf16 ? 2 : 4);
        const int64_t tt = c0 + tid;
        // Element offsets within each tensor (checked in a bounds build).
        const int64_t o_dt = b * p.sdt[0] + h * p.sdt[1], o_adt = b * p.sadt[0] + h * p.sadt[1];
        const int64_t o_tr = b * p.str[0] + h * p.str[1];
        auto trap_at = [&](int64_t x) { return tf_in(o_tr + x, 1, p.ext_trap) ? load_trap(p, trbase, x) : 0.f; };
        if (kExt && p.raw_controls) {
          // dt = softplus(ddt + dt_bias), adt = A dt from the projection views.
          const int64_t o_a = b * p.sar[0] + h * p.sar[2], o_d = b * p.sdr[0] + h * p.sdr[2];
          const bf16* abase = p.a_raw + b * p.sar[0] + h * p.sar[2];
          const bf16* dbase = p.ddt_raw + b * p.sdr[0] + h * p.sdr[2];
          auto a_at = [&](int64_t x) { return tf_in(o_a + x, 1, p.ext_ar) ? bf2f(abase[x]) : 0.f; };
          auto d_at = [&](int64_t x) { return tf_in(o_d + x, 1, p.ext_dr) ? bf2f(dbase[x]) : 0.f; };
          const float bias = tf_in(h, 1, p.H) ? p.dt_bias[h] : 0.f;
          if (tid < nv) {
            const int64_t sr = src_row(tt);
            c_dt = softplus_dt(d_at(sr * p.sdr[1]) + bias);
            c_adt = a_control(a_at(sr * p.sar[1]), p.a_floor) * c_dt;
            c_tr = trap_at(sr * p.str[2]);
          }
          if (tt + 1 < T_eff) {
            const int64_t sn = src_row(tt + 1);
            c_dn = softplus_dt(d_at(sn * p.sdr[1]) + bias);
            c_tn = trap_at(sn * p.str[2]);
          }
        } else {
          auto dt_at = [&](int64_t x) { return tf_in(o_dt + x, 1, p.ext_dt) ? dtbase[x] : 0.f; };
          if (tid < nv) {
            const int64_t sr = src_row(tt);
            c_dt = dt_at(sr * p.sdt[2]);
            c_tr = trap_at(sr * p.str[2]);
            c_adt = tf_in(o_adt + sr * p.sadt[2], 1, p.ext_adt) ? adtbase[sr * p.sadt[2]] : 0.f;
          }
          if (tt + 1 < T_eff) {
            const int64_t sn = src_row(tt + 1);
            c_dn = dt_at(sn * p.sdt[2]);
            c_tn = trap_at(sn * p.str[2]);
          }
        }
      }
      float araw[8];
      if (tma_rows) {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int tt = warp * 8 + i, ra = rev ? kChunk - 1 - tt : tt;
          araw[i] = tt < nv ? __uint_as_float(ld_shared_u16(stage + kStA + ra * 64u + lane * 2u) << 16) : 0.f;
        }
      } else if (kStage && p.ang_vec) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          araw[i] = __uint_as_float(ld_shared_u16(stage + kStA + (warp * 8 + i) * 64u + lane * 2u) << 16);
      } else {
        const bf16* abase = p.ang + b * p.sa[0] + h * p.sa[2];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int tt = warp * 8 + i;
          const int64_t ax = src_row(c0 + tt) * p.sa[1] + lane * p.sa[3];
          araw[i] = (tt < nv && tf_in(b * p.sa[0] + h * p.sa[2] + ax, 1, p.ext_a)) ? bf2f(abase[ax]) : 0.f;
        }
      }
      // The slot's previous unit must be fully retired before it is rewritten.
      if (k >= 2) ok &= mbar_wait(&mi.freed[slot], ((k >> 1) - 1) & 1);
      const uint32_t sb = base + slot * kSlotBytes;
      // ---- controls and the decay cumsum ----------------------------------------
      if (tid < kChunk) {
        const float gm = c_dt * sigmoidf_fast(c_tr);
        float x = c_adt * kLog2e;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float y = __shfl_up_sync(0xffffffffu, x, o);
          if (lane >= o) x += y;
        }
        if (lane == 31) mi.wsum[warp] = x;
        mi.dtc[tid] = c_dt;
        const float scl = c_dn * (1.f - sigmoidf_fast(c_tn)) + gm;
        mi.scale[tid] = scl;
        hd.g[tid] = scl > 0.f ? gm * rcp_approx(scl) : 0.f;
        hd.cs[tid] = x;
      }
      if (!kLook && tid == kClaimThread) mi.next_ticket = my_next;
      bar_sync_n(kBarProducer, kProducerThreads);  // also: every thread has read its staged rows
      if constexpr (!kLook) stage_unit(mi.next_ticket);
      if (tid < kChunk) {
        // Final cumsum, and its range over the chunk (warps 0-1).
        float cv = hd.cs[tid];
        if (tid >= 32) {
          cv += mi.wsum[0];
          hd.cs[tid] = cv;
        }
        float hi = cv, lo = cv;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
          lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
        }
        if (lane == 0) {
          mi.csmax[warp] = hi;
          mi.csmin[warp] = lo;
        }
      }
      // ---- local angle phases: lane = pair r, warp = 8-step segment ------------
      float* phase = reinterpret_cast<float*>(smem + kOffPhase);
      {
        float run = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const int tt = warp * 8 + i;
          run = fmaf(tanh_approx(araw[i]) * kPi, mi.dtc[tt], run);
          phase[tt * 33 + lane] = run;
        }
        mi.seg[warp][lane] = run;
      }
      bar_sync_n(kBarProducer, kProducerThreads);
      {
        float off = 0.f;
        for (int q = 0; q < warp; ++q) off += mi.seg[q][lane];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float ph = phase[(warp * 8 + i) * 33 + lane] + off;
          phase[(warp * 8 + i) * 33 + lane] = ph - kTwoPi * floorf(ph * (1.f / kTwoPi));
        }
        if (warp == 0) {
          float th = 0.f;
#pragma unroll
          for (int q = 0; q < 8; ++q) th += mi.seg[q][lane];
          hd.theta[lane] = th - kTwoPi * floorf(th * (1.f / kTwoPi));
        }
      }
      bar_sync_n(kBarProducer, kProducerThreads);
      // Long rows: the next unit is claimed here and staged at the end of the iteration.
      if (kLook && tid == kClaimThread && held < quota) my_next = ticket_unit(atomicAdd(ws_ticket, 1));
      const float total = hd.cs[kChunk - 1];
      // Decay reference of the unit: mu near the middle of the cumsum's range, with
      // E = total - mu an integer, so that the decay-weighted values vs below are
      // exact power-of-two multiples of v.
      const float cmax = fmaxf(mi.csmax[0], mi.csmax[1]), cmin = fminf(mi.csmin[0], mi.csmin[1]);
      const float Ef = rintf(total - 0.5f * (cmax + cmin));
      const float mu = total - Ef;
      // Over 180 binades of decay in one chunk: P's row and column factors would leave
      // FP32's range, so the epilogue combines them per element.
      const bool wide = cmax - cmin > 180.f;
      // ---- rows -> FP16 operand tiles (q16, k~, vs, v16) and the z tile ------------
      {
        const int hb = TF_OFF(tf_in(static_cast<int64_t>(h) * kState, kState, static_cast<int64_t>(p.H) * kState), h);
        const float* qbh = p.qb + hb * kState;
        const float* kbh = p.kb + hb * kState;
        float cn[8], sn[8];  // this thread's 8 rotating pairs: 4s..4s+3, 16+4s..16+4s+3
#pragma unroll
        for (int m = 0; m < 8; ++m)
          __sincosf(phase[t * 33 + (m < 4 ? 4 * s4 + m : 12 + 4 * s4 + m)], &sn[m], &cn[m]);
        float x[32];
        // q: optional C_norm, bias, rotation, row exponent.
        const float qmax = prep_qk_row(x, qraw, p.qw, p.eps, qbh, s4, cn, sn);
        const int qe = pow2_scale_exponent(qmax);
        {
          const float qs = exp2i(qe);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int e0 = 32 * i + 8 * s4;
            st_shared_v4(sb + kSlotQ + (e0 >> 6) * 8192u + sw128_offset(t, e0 & 63),
                         pack_f16x2(x[8 * i] * qs, x[8 * i + 1] * qs), pack_f16x2(x[8 * i + 2] * qs, x[8 * i + 3] * qs),
                         pack_f16x2(x[8 * i + 4] * qs, x[8 * i + 5] * qs),
                         pack_f16x2(x[8 * i + 6] * qs, x[8 * i + 7] * qs));
          }
        }
        // k: optional B_norm, bias, rotation.
        const float kmax = prep_qk_row(x, kraw, p.kw, p.eps, kbh, s4, cn, sn);
        float vf[16];
        unpack8(vraw[0], &vf[0]);
        unpack8(vraw[1], &vf[8]);
        float vmax = 0.f;
#pragma unroll
        for (int e = 0; e < 16; ++e) vmax = fmaxf(vmax, fabsf(vf[e]));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 1));
        vmax = fmaxf(vmax, __shfl_xor_sync(0xffffffffu, vmax, 2));
        // Key j's weight scale_j 2^(mu - cs_j) goes into the k row as scale_j 2^(d_j),
        // with d_j = mu - cs_j - n_j, n_j an integer that is 0 unless |mu - cs_j| > 100
        // (wide units); 2^(E + n_j) goes into vs. Then the state contribution is
        //   k~_j^T vs_j = kr_j scale_j 2^(total - cs_j) v_j
        // and the scores q16_i . k~_j carry 2^(qe_i + ke_j + d_j) besides the decay.
        const float tj = mu - hd.cs[t];
        const float nj = tj > 100.f ? floorf(tj - 100.f) : (tj < -100.f ? -floorf(-tj - 100.f) : 0.f);
        const float kf0 = row_ok ? mi.scale[t] * ex2_approx(tj - nj) : 0.f;
        // Split the remaining power of two between k~ = kr kf0 2^ke and vs = v 2^(E+n_j-ke)
        // near the geometric mean of their magnitudes, but keep the k~ row maximum >= 2^-6
        // so the scores keep FP16's full precision; a vs row pushed below that carries a
        // negligible state contribution. Both stay below 2^15.
        const int kl = ilog2_or(kmax * kf0, 1000);
        const int vl = vmax > 0.f ? ilog2_or(vmax, 0) + static_cast<int>(Ef + nj) : 1000;
        int ke = 0;
        if (kl != 1000) {
          ke = vl != 1000 ? ((vl - kl) >> 1) : 14 - kl;
          ke = max(ke, -6 - kl);
          if (vl != 1000) ke = max(ke, vl - 14);
          ke = min(ke, 14 - kl);
          ke = ke < -120 ? -120 : (ke > 120 ? 120 : ke);
        }
        {
          const float kf = kf0 * exp2i(ke);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const int e0 = 32 * i + 8 * s4;
            st_shared_v4(sb + kSlotK + (e0 >> 6) * 8192u + sw128_offset(t, e0 & 63),
                         pack_f16x2(x[8 * i] * kf, x[8 * i + 1] * kf), pack_f16x2(x[8 * i + 2] * kf, x[8 * i + 3] * kf),
                         pack_f16x2(x[8 * i + 4] * kf, x[8 * i + 5] * kf),
                         pack_f16x2(x[8 * i + 6] * kf, x[8 * i + 7] * kf));
          }
          // vs = v 2^(E + n_j - ke): an exact power-of-two multiple of the BF16 v while it
          // stays in FP16's normal range (zero below 2^-126 and for rows past the length).
          const int ev = static_cast<int>(Ef + nj) - ke;
          const float vsc = (row_ok && ev >= -126) ? exp2i(ev > 127 ? 127 : ev) : 0.f;
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const uint32_t off = sw128_offset(t, 32 * i + 8 * s4);
            uint32_t hv[4], hs[4];
#pragma unroll
            for (int m = 0; m < 4; ++m) {
              const float a0 = row_ok ? vf[8 * i + 2 * m] : 0.f, a1 = row_ok ? vf[8 * i + 2 * m + 1] : 0.f;
              hv[m] = pack_f16x2(a0, a1);
              hs[m] = pack_f16x2(a0 * vsc, a1 * vsc);
            }
            st_shared_v4(sb + kSlotV + off, hv[0], hv[1], hv[2], hv[3]);
            st_shared_v4(sb + kSlotVS + off, hs[0], hs[1], hs[2], hs[3]);
            st_shared_v4(sb + kSlotZ + off, zraw[i].x, zraw[i].y, zraw[i].z, zraw[i].w);
          }
        }
        if (s4 == 0) {
          // P_ij = D_ij 2^(cl_j) 2^(rl_i) for j < i, with D the score accumulator.
          const float cl = nj - static_cast<float>(ke);
          hd.qe[t] = static_cast<float>(qe);
          const float rl = hd.cs[t] - mu - static_cast<float>(qe);
          hd.rl[t] = wide ? rl : fminf(fmaxf(rl, -126.f), 126.f);  // (bounded unless q rows are extreme)
          hd.cl[t] = cl;
          hd.cf[t] = exp2i(cl < -126.f ? -126 : (cl > 127.f ? 127 : static_cast<int>(cl)));
        }
      }
      if (tid == 0) {
        hd.unit = u;
        hd.b = b;
        hd.h = h;
        hd.c = c;
        hd.nv = nv;
        hd.dir = dir;
        hd.teff = T_eff;
        hd.gtot = ex2_approx(total);
        hd.wide = wide ? 1 : 0;
      }
      if (kLook && tid == kClaimThread) mi.next_ticket = my_next;
      fence_async_smem();
      tc_fence_before();
      bar_sync_n(kBarProducer, kProducerThreads);
      if constexpr (kLook) stage_unit(mi.next_ticket);
      pend = slot;  // MMA 1 is issued at the top of the next iteration
      if (mi.next_ticket >= shp.units) {
        // No next unit: issue it now (nothing in this CTA waits behind warp 6 any more).
        if (tid == kMmaThread) issue_mma1(pend);
        pend = -1;
      }
      ++k;
    }
    // Units wholly past their row's length: zero their output rows. A static
    // share per CTA (no waits involved), so no ticket has to reach them.
    for (int zu = blockIdx.x; zu < shp.units; zu += gridDim.x) {
      int zb, zh, zc, zd;
      decode_unit(zu, shp, zb, zh, zc, zd);
      if (kDirs == 1) zd = 0;
      const RecurrenceParams& pz = (kDirs == 1 || zd == 0) ? pd0 : pd1;
      const int z0 = zc * kChunk;
      if (z0 < teff_of(zd, zb, pz) || z0 + t >= pz.T) continue;
      const int64_t oz = zb * pz.so[0] + static_cast<int64_t>(z0 + t) * pz.so[1] + zh * pz.so[2];
      if (!tf_in(oz, kHead, pz.ext_out)) continue;
      bf16* orow = pz.out + oz;
#pragma unroll
      for (int i = 0; i < 2; ++i) store16<kVec>(orow + 32 * i + 8 * s4, make_uint4(0, 0, 0, 0));
    }
  } else {
    // =========================== epilogue ===========================
    const int et = tid - kProducerThreads;  // 0..255
    const int q4 = warp & 3;                // TMEM lane quarter
    const int chalf = (warp - 8) >> 2;      // 32-column half
    const int g = lane >> 2, c4 = lane & 3;
    const int i0 = 16 * q4 + g, i1 = i0 + 8;   // rows of the M=64 accumulators
    const uint32_t n = 32 * q4 + lane;          // row of the M=128 accumulator / state
    for (int k = 0;; ++k) {
      const int slot = k & 1;
      const uint32_t ph = (k >> 1) & 1;
      SlotHeader& hd = mi.hdr[slot];
      ok &= mbar_wait(&mi.ready[slot], ph);
      const int u = hd.unit;
      if (u < 0) break;
      const int b = hd.b, h = hd.h, c = hd.c, dir = kDirs == 1 ? 0 : hd.dir;
      const RecurrenceParams& p = (kDirs == 1 || dir == 0) ? pd0 : pd1;
      const uint32_t sb = base + slot * kSlotBytes;
      const uint32_t tm = tmem0 + slot * kSlotCols;
      unsigned char* uws = uws_of(u);
      ok &= mbar_wait(&mi.mma1[slot], ph);
      tc_fence_after();
      // The row's last chunk has no successor: nothing reads its dS, flag or state.
      // (Read from the slot header at each use rather than held in a register.)
      auto last = [&]() { return (c + 1) * kChunk >= hd.teff; };
      // ---- export dS^T (row n, this thread's 32-column half) -----------------------
      if (!last()) {
        float r[32];
        tmem_ld16(tmem_addr(tm, 32 * q4, kColD + 32 * chalf), *reinterpret_cast<float(*)[16]>(&r[0]));
        tmem_ld16(tmem_addr(tm, 32 * q4, kColD + 32 * chalf + 16), *reinterpret_cast<float(*)[16]>(&r[16]));
        tmem_wait_ld();
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) m = fmaxf(m, fabsf(r[j]));
        const int ae = pow2_scale_exponent(m);
        const float as = exp2i(ae);
        __half* agg = reinterpret_cast<__half*>(uws + kUnitAgg) + n * 64 + 32 * chalf;
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float* rr = &r[8 * q];
          *reinterpret_cast<uint4*>(agg + 8 * q) =
              make_uint4(pack_f16x2(rr[0] * as, rr[1] * as), pack_f16x2(rr[2] * as, rr[3] * as),
                         pack_f16x2(rr[4] * as, rr[5] * as), pack_f16x2(rr[6] * as, rr[7] * as));
        }
        reinterpret_cast<float*>(uws + kUnitExp)[128 * chalf + n] = exp2i(-ae);
        if (et < kRotary) reinterpret_cast<float*>(uws + kUnitTheta)[et] = hd.theta[et];
        if (et == 0) reinterpret_cast<float*>(uws + kUnitTheta)[kRotary] = hd.gtot;
      }
      // ---- helpers of the state fold (row n, this thread's 32-column half) ----------
      // One step: st = R(-theta) (g st + dS), dS from a published unit.
      auto fold_step = [&](float (&st)[32], const uint4 (&w)[4], float f, float gx, float th) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint32_t ww[4] = {w[q].x, w[q].y, w[q].z, w[q].w};
#pragma unroll
          for (int mm = 0; mm < 4; ++mm) {
            const float2 v = unpack_f16x2(ww[mm]);
            st[8 * q + 2 * mm] = fmaf(gx, st[8 * q + 2 * mm], v.x * f);
            st[8 * q + 2 * mm + 1] = fmaf(gx, st[8 * q + 2 * mm + 1], v.y * f);
          }
        }
        if (q4 < 2) {  // rows n < 64 hold the 32 rotating pairs (2r, 2r+1)
          float snx, cnx;
          __sincosf(th, &snx, &cnx);
          const float sgn = (n & 1u) ? -snx : snx;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float other = __shfl_xor_sync(0xffffffffu, st[j], 1);
            st[j] = fmaf(st[j], cnx, other * sgn);  // R(-theta)
          }
        }
      };
      // This unit's own published dS (row n, this thread's half), rebuilt from the
      // accumulator still in TMEM with the export's exponent and rounding, so it is
      // bit for bit what successors read from the workspace (no L2 round trip).
      auto own_ds = [&](uint4 (&w)[4], float& f) {
        float r[32];
        tmem_ld16(tmem_addr(tm, 32 * q4, kColD + 32 * chalf), *reinterpret_cast<float(*)[16]>(&r[0]));
        tmem_ld16(tmem_addr(tm, 32 * q4, kColD + 32 * chalf + 16), *reinterpret_cast<float(*)[16]>(&r[16]));
        tmem_wait_ld();
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) m = fmaxf(m, fabsf(r[j]));
        const int ae = pow2_scale_exponent(m);
        const float as = exp2i(ae);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float* rr = &r[8 * q];
          w[q] = make_uint4(pack_f16x2(rr[0] * as, rr[1] * as), pack_f16x2(rr[2] * as, rr[3] * as),
                            pack_f16x2(rr[4] * as, rr[5] * as), pack_f16x2(rr[6] * as, rr[7] * as));
        }
        f = exp2i(-ae);
      };
      // Loads of a predecessor whose dS is known to be published.
      auto fetch = [&](int x, uint4 (&w)[4], float& f, float& gx, float& th) {
        const unsigned char* xws = uws_of(unit_index(shp, x, dir, b, h));
        const __half* agg = reinterpret_cast<const __half*>(xws + kUnitAgg) + n * 64 + 32 * chalf;
#pragma unroll
        for (int q = 0; q < 4; ++q) w[q] = ld_cg_v4(agg + 8 * q);
        f = __ldcg(reinterpret_cast<const float*>(xws + kUnitExp) + 128 * chalf + n);
        gx = __ldcg(reinterpret_cast<const float*>(xws + kUnitTheta) + kRotary);
        th = __ldcg(reinterpret_cast<const float*>(xws + kUnitTheta) + ((n >> 1) & 31u));
      };
      // The state entering chunk c (c > 0): predecessors' contributions folded from the
      // nearest published outgoing state (look-back rows) or from chunk 0.
      float st[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) st[j] = 0.f;
      auto fold_predecessors = [&]() {
        int start = 0;
        if (lookback) {
          // Nearest predecessor y with a published outgoing state such that every unit
          // after it has published its dS (y = -1: none, start from chunk 0). One warp
          // reads the flags of 32 predecessors at once (lane l: chunk base - l) and
          // re-reads the window until the nearest published state is reached through
          // published dS; a window of published dS without a state moves 32 chunks back.
          if (et < 32) {
            int base = c - 1, y = -1;
            const uint64_t t0 = global_timer_ns();
            for (;;) {
              const int x = base - lane;
              int rel = static_cast<int>(kFlagIncl);  // chunk -1 acts as a published zero state
              if (x >= 0)
                rel = static_cast<int>(
                    ld_acquire_u32(reinterpret_cast<const uint32_t*>(uws_of(unit_index(shp, x, dir, b, h)) + kUnitFlag)) -
                    epoch);
              const uint32_t incl = __ballot_sync(0xffffffffu, x < 0 || rel >= static_cast<int>(kFlagIncl));
              const uint32_t agg = __ballot_sync(0xffffffffu, x < 0 || rel >= static_cast<int>(kFlagAgg));
              if (incl) {
                const int j = __ffs(static_cast<int>(incl)) - 1;  // nearest published state
                const uint32_t need = (1u << j) - 1u;              // the dS after it
                if ((agg & need) == need) {
                  y = base - j;
                  break;
                }
              } else if (agg == 0xffffffffu) {
                base -= 32;
                continue;
              }
              if (global_timer_ns() - t0 > p0.flag_wait_ns) {
                ok = false;
                y = -1;
                break;
              }
              __nanosleep(64);
            }
            if (lane == 0) mi.lookback_start = y;
          }
          bar_sync_n(kBarEpilogue, kEpilogueThreads);
          const int y = mi.lookback_start;
          if (y >= 0) {
            const unsigned char* yws = uws_of(unit_index(shp, y, dir, b, h));
            (void)ld_acquire_u32(reinterpret_cast<const uint32_t*>(yws + kUnitFlag));
            const float* incl = reinterpret_cast<const float*>(yws + kUnitIncl) + n * 64 + 32 * chalf;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const uint4 w = ld_cg_v4(incl + 4 * q);
              st[4 * q] = __uint_as_float(w.x);
              st[4 * q + 1] = __uint_as_float(w.y);
              st[4 * q + 2] = __uint_as_float(w.z);
              st[4 * q + 3] = __uint_as_float(w.w);
            }
            start = y + 1;
          }
        } else {
          // Short rows: lane l of every warp waits for predecessor l's dS flag.
          for (int x = lane; x < c; x += 32) {
            uint32_t seen = 0;
            ok &= wait_flag(reinterpret_cast<const uint32_t*>(uws_of(unit_index(shp, x, dir, b, h)) + kUnitFlag),
                            epoch, kFlagAgg, seen, p0.flag_wait_ns);
          }
          __syncwarp();
        }
        if (start < c) {
          uint4 wa[4];
          float fa, ga, ta;
          fetch(start, wa, fa, ga, ta);
          for (int x = start; x < c; ++x) {
            uint4 wb[4];
            float fb = 0.f, gb = 0.f, tb = 0.f;
            if (x + 1 < c) fetch(x + 1, wb, fb, gb, tb);  // in flight while x is folded
            fold_step(st, wa, fa, ga, ta);
#pragma unroll
            for (int q = 0; q < 4; ++q) wa[q] = wb[q];
            fa = fb;
            ga = gb;
            ta = tb;
          }
        }
      };
      if (lookback) {
        // Rows of many chunks: the chain of outgoing states along the row sets the
        // launch's time, so this unit's link in it (dS flag, fold, outgoing state)
        // comes before its own output work. Every epilogue thread's export stores
        // precede this barrier, and a release after a CTA barrier is cumulative over
        // them, so one thread's gpu-scope release orders the whole export before the flag.
        bar_sync_n(kBarEpilogue, kEpilogueThreads);
        if (et == kEpilogueThreads - 32 && !last())
          st_release_u32(reinterpret_cast<uint32_t*>(uws + kUnitFlag), epoch + kFlagAgg);
        if (c > 0) fold_predecessors();
        if (!last()) {
          // Outgoing state S(c+1) = R(-theta_c) (2^total_c S(c) + dS_c).
          float so[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) so[j] = st[j];
          uint4 w[4];
          float f;
          own_ds(w, f);
          fold_step(so, w, f, hd.gtot, hd.theta[(n >> 1) & 31u]);
          float* incl = reinterpret_cast<float*>(uws + kUnitIncl) + n * 64 + 32 * chalf;
#pragma unroll
          for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(incl + 4 * q) = make_float4(so[4 * q], so[4 * q + 1], so[4 * q + 2], so[4 * q + 3]);
          bar_sync_n(kBarEpilogue, kEpilogueThreads);  // the release below is cumulative over these stores
          if (et == 0) st_release_u32(reinterpret_cast<uint32_t*>(uws + kUnitFlag), epoch + kFlagIncl);
        }
      }
      // ---- decayed scores P (+ the D-skip diagonal) -> FP16 hi/lo tiles ---------
      // P_ij = D_ij 2^(cl_j) 2^(rl_i) for j < i (D the score accumulator: the decay is
      // split between the k~ rows and these factors), d + P_ii g_i on the diagonal.
      {
        // Warps whose 16 rows (< 32) all lie above their 32 columns (>= 32) hold zeros.
        const bool upper = q4 < 2 && chalf == 1;
        float sc[16];
        float m0 = 0.f, m1 = 0.f;
        if (!upper) {
          tmem_ld_16x256_x4(tmem_addr(tm, 32 * q4, kColS + 32 * chalf), sc);
          tmem_wait_ld();
          const float d = tf_in(h, 1, p.H) ? p.d[h] : 0.f;
          const float g0 = hd.g[i0], g1 = hd.g[i1];
          const float rl0 = hd.rl[i0], rl1 = hd.rl[i1];
          const bool wide_u = hd.wide != 0;
          const float r0 = ex2_approx(rl0), r1 = ex2_approx(rl1);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              const int j = 32 * chalf + 8 * kk + 2 * c4 + e;
              float v0 = sc[4 * kk + e], v1 = sc[4 * kk + 2 + e];
              if (!wide_u) {
                const float cf = hd.cf[j];
                v0 = (v0 * cf) * r0;
                v1 = (v1 * cf) * r1;
              } else {
                const float cl = hd.cl[j];
                v0 *= ex2_approx(rl0 + cl);
                v1 *= ex2_approx(rl1 + cl);
              }
              v0 = j < i0 ? v0 : (j == i0 ? fmaf(v0, g0, d) : 0.f);
              v1 = j < i1 ? v1 : (j == i1 ? fmaf(v1, g1, d) : 0.f);
              sc[4 * kk + e] = v0;
              sc[4 * kk + 2 + e] = v1;
              m0 = fmaxf(m0, fabsf(v0));
              m1 = fmaxf(m1, fabsf(v1));
            }
          }
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) sc[e] = 0.f;
        }
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 1));
        m0 = fmaxf(m0, __shfl_xor_sync(0xffffffffu, m0, 2));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 1));
        m1 = fmaxf(m1, __shfl_xor_sync(0xffffffffu, m1, 2));
        if (c4 == 0) {
          hd.pmax[chalf][i0] = m0;
          hd.pmax[chalf][i1] = m1;
        }
        bar_sync_n(kBarPair + q4, 64);  // the two warps sharing this TMEM quarter
        m0 = fmaxf(hd.pmax[0][i0], hd.pmax[1][i0]);
        m1 = fmaxf(hd.pmax[0][i1], hd.pmax[1][i1]);
        const int pe0 = pow2_scale_exponent(m0), pe1 = pow2_scale_exponent(m1);
        if (chalf == 0 && c4 == 0) {
          hd.pe[i0] = static_cast<float>(pe0);
          hd.pe[i1] = static_cast<float>(pe1);
        }
        const float ps0 = exp2i(pe0), ps1 = exp2i(pe1);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int j = 32 * chalf + 8 * kk + 2 * c4;
          const float a0 = sc[4 * kk] * ps0, a1 = sc[4 * kk + 1] * ps0;
          const float b0 = sc[4 * kk + 2] * ps1, b1 = sc[4 * kk + 3] * ps1;
          const uint32_t h0 = pack_f16x2(a0, a1), h1 = pack_f16x2(b0, b1);
          const float2 f0 = unpack_f16x2(h0), f1 = unpack_f16x2(h1);
          st_shared_u32(sb + kSlotPH + sw128_offset(i0, j), h0);
          st_shared_u32(sb + kSlotPH + sw128_offset(i1, j), h1);
          st_shared_u32(sb + kSlotPL + sw128_offset(i0, j), pack_f16x2(a0 - f0.x, a1 - f0.y));
          st_shared_u32(sb + kSlotPL + sw128_offset(i1, j), pack_f16x2(b0 - f1.x, b1 - f1.y));
        }
      }
      fence_async_smem();
      tc_fence_before();
      bar_sync_n(kBarEpilogue, kEpilogueThreads);
      if (et == 0) {
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tm + kColPV, desc_sw128(sb + kSlotPH + kk * 32u, 0, 1024),
                   desc_sw128(sb + kSlotV + kk * 2048u, 8192, 1024), kIdPV, kk > 0);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tm + kColPV, desc_sw128(sb + kSlotPL + kk * 32u, 0, 1024),
                   desc_sw128(sb + kSlotV + kk * 2048u, 8192, 1024), kIdPV, 1);
        umma_commit(&mi.mma2[slot]);
      }
      if (!lookback) {
        // Publish dS (a thread of warp 15, in parallel with warp 8's MMA issue). Every
        // epilogue thread's export stores precede the barrier above, and a release
        // after a CTA barrier is cumulative over them, so one thread's gpu-scope
        // release orders the whole export before the flag.
        if (et == kEpilogueThreads - 32 && !last())
          st_release_u32(reinterpret_cast<uint32_t*>(uws + kUnitFlag), epoch + kFlagAgg);
        if (c > 0) fold_predecessors();
      }
      if (c > 0) {
        // FP16 S^T tile with one power-of-two exponent: this thread's part of the maximum.
        float m = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) m = fmaxf(m, fabsf(st[j]));
        m = warp_max(m);
        if (lane == 0) mi.ered[warp - 8] = m;
        // The S^T tile overwrites vs and v16: MMA 2, the last reader of v16, must be done.
        ok &= mbar_wait(&mi.mma2[slot], ph);
        bar_sync_n(kBarEpilogue, kEpilogueThreads);  // the maxima
#pragma unroll
        for (int w8 = 0; w8 < 8; ++w8) m = fmaxf(m, mi.ered[w8]);
        const int se = pow2_scale_exponent(m);
        const float ss = exp2i(se);
        if (et == 0) hd.sinv = exp2i(-se);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          st_shared_v4(sb + kSlotS + sw128_offset(n, 32 * chalf + 8 * q), pack_f16x2(st[8 * q] * ss, st[8 * q + 1] * ss),
                       pack_f16x2(st[8 * q + 2] * ss, st[8 * q + 3] * ss), pack_f16x2(st[8 * q + 4] * ss, st[8 * q + 5] * ss),
                       pack_f16x2(st[8 * q + 6] * ss, st[8 * q + 7] * ss));
        fence_async_smem();
        tc_fence_before();
        bar_sync_n(kBarEpilogue, kEpilogueThreads);
        if (et == 0) {
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint32_t koff = (kk >> 2) * 8192u + (kk & 3) * 32u;
            umma_f16(tm + kColI, desc_sw128(sb + kSlotQ + koff, 0, 1024),
                     desc_sw128(sb + kSlotS + kk * 2048u, 8192, 1024), kIdInter, kk > 0);
          }
          umma_commit(&mi.mma3[slot]);
        }
      } else {
        if (et == 0) mbar_arrive(&mi.mma3[slot]);  // no inter-chunk MMA; keep the phase in step
      }
      // ---- output: combine, gate, stage in the z tile, coalesced stores ----------
      ok &= mbar_wait(&mi.mma2[slot], ph);
      ok &= mbar_wait(&mi.mma3[slot], ph);
      tc_fence_after();
      {
        float pv[16], it[16];
        tmem_ld_16x256_x4(tmem_addr(tm, 32 * q4, kColPV + 32 * chalf), pv);
        if (c > 0) tmem_ld_16x256_x4(tmem_addr(tm, 32 * q4, kColI + 32 * chalf), it);
        tmem_wait_ld();
        const float u0 = exp2i(-static_cast<int>(hd.pe[i0])), u1 = exp2i(-static_cast<int>(hd.pe[i1]));
        const float w0 = c > 0 ? ex2_approx(hd.cs[i0] - hd.qe[i0]) * hd.sinv : 0.f;
        const float w1 = c > 0 ? ex2_approx(hd.cs[i1] - hd.qe[i1]) * hd.sinv : 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          const int j = 32 * chalf + 8 * kk + 2 * c4;
          const uint32_t a0 = sb + kSlotZ + sw128_offset(i0, j), a1 = sb + kSlotZ + sw128_offset(i1, j);
          const float2 z0 = unpack_bf16x2(ld_shared_u32(a0)), z1 = unpack_bf16x2(ld_shared_u32(a1));
          const float o0 = pv[4 * kk] * u0 + (c > 0 ? it[4 * kk] * w0 : 0.f);
          const float o1 = pv[4 * kk + 1] * u0 + (c > 0 ? it[4 * kk + 1] * w0 : 0.f);
          const float o2 = pv[4 * kk + 2] * u1 + (c > 0 ? it[4 * kk + 2] * w1 : 0.f);
          const float o3 = pv[4 * kk + 3] * u1 + (c > 0 ? it[4 * kk + 3] * w1 : 0.f);
          st_shared_u32(a0, pack_bf16x2(o0 * silu_tanh(z0.x), o1 * silu_tanh(z0.y)));
          st_shared_u32(a1, pack_bf16x2(o2 * silu_tanh(z1.x), o3 * silu_tanh(z1.y)));
        }
      }
      tc_fence_before();
      bar_sync_n(kBarEpilogue, kEpilogueThreads);
      {
        const int c0 = c * kChunk, nv = hd.nv;
        // 64 rows x 8 16-byte chunks over 256 threads: row et/4, chunks 2*(et&3), +1.
        const int r = et >> 2;
        if (c0 + r < p.T) {
          // Valid rows of a reversed row go back to time len-1-x; padding stays put.
          const int64_t row = (kExt && p.reverse && r < nv) ? static_cast<int64_t>(hd.teff - 1 - (c0 + r)) : c0 + r;
          const int64_t oo = b * p.so[0] + row * p.so[1] + h * p.so[2];
          if (tf_in(oo, kHead, p.ext_out)) {  // (a bounds build skips an out-of-range row)
            bf16* orow = p.out + oo;
#pragma unroll
            for (int q = 0; q < 2; ++q) {
              const int e = 8 * (2 * (et & 3) + q);
              const uint4 val = r < nv ? ld_shared_v4(sb + kSlotZ + sw128_offset(r, e)) : make_uint4(0, 0, 0, 0);
              store16<kVec>(orow + e, val);
            }
          }
        }
      }
      bar_sync_n(kBarEpilogue, kEpilogueThreads);
      if (et == 0) mbar_arrive(&mi.freed[slot]);
    }
  }

  // ---- teardown: free TMEM; the last CTA advances the epoch -----------------------
  if (!ok) {
    atomicExch(&g_device_error, 1);
    if (p0.err_host) {  // a plain store: host memory over PCIe need not support atomics
      *reinterpret_cast<volatile int*>(p0.err_host) = 1;
      __threadfence_system();
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem0, kTmemCols);
  }
  if (tid == 0) {
    // One ordering point: the release half orders this CTA's ticket claims
    // (same thread) before its count, and the acquire half lets the last CTA
    // see every other CTA's claims before it resets the counters. What the next
    // launch reads (counters, epoch) is ordered by the kernel boundary itself.
    if (atom_add_acq_rel(ws_done, 1) == static_cast<int>(gridDim.x) - 1) {
      *reinterpret_cast<volatile int*>(ws_ticket) = 0;
      *reinterpret_cast<volatile int*>(ws_done) = 0;
      *reinterpret_cast<volatile uint32_t*>(ws_epoch) = epoch + kEpochStep;
    }
  }
}

// One direction: a single parameter block (the launch copies less). kLook: rows
// of more than kLookbackChunks chunks (outgoing states and look-back compiled in).
template <int kVec, bool kExt, bool kLook, bool kTma>
__global__ void __launch_bounds__(kThreads, 1) recurrence_persistent_kernel(const __grid_constant__ RecurrenceParams p,
                                                                              unsigned char* ws) {
  recurrence_body<kVec, 1, kExt, kLook, kTma>(p, p, ws);
}
// Both directions of a bidirectional pair in one launch.
template <int kVec, bool kLook, bool kTma>
__global__ void __launch_bounds__(kThreads, 1) recurrence_pair_kernel(const __grid_constant__ RecurrenceParams p0,
                                                                        const __grid_constant__ RecurrenceParams p1,
                                                                        unsigned char* ws) {
  recurrence_body<kVec, 2, true, kLook, kTma>(p0, p1, ws);
}

int alignment_class_one(const RecurrenceParams& p) {
  auto rows_aligned = [](const void* ptr, const int64_t* st, int nd, int bytes) {
    if (reinterpret_cast<uintptr_t>(ptr) % bytes) return false;
    for (int i = 0; i < nd; ++i)
      if ((st[i] * 2) % bytes) return false;
    return true;
  };
  for (int bytes : {16, 8}) {
    if (rows_aligned(p.q, p.sq, 3, bytes) && rows_aligned(p.k, p.sk, 3, bytes) &&
        rows_aligned(p.v, p.sv, 3, bytes) && rows_aligned(p.z, p.sz, 3, bytes) &&
        rows_aligned(p.out, p.so, 3, bytes))
      return bytes;
  }
  return 2;
}

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices] = {0};

int sm_count() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return 148;
  if (g_sm_count[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = n > 0 ? n : 148;
  }
  return g_sm_count[dev];
}

// Angle rows can be staged with 8-byte cp.async: aligned rows of contiguous pairs.
int angles_vectorizable(const RecurrenceParams& p) {
  if (reinterpret_cast<uintptr_t>(p.ang) % 8 || p.sa[3] != 1) return 0;
  for (int i = 0; i < 3; ++i)
    if ((p.sa[i] * 2) % 8) return 0;
  return 1;
}

// ---- tensor maps for the TMA staging of a unit's rows --------------------------
PFN_cuTensorMapEncodeTiled_v12000 g_encode_tiled = nullptr;
int g_encode_state = 0;  // 0: not looked up, 1: available, 2: unavailable

bool encode_available() {
  if (g_encode_state == 0) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (e == cudaSuccess && q == cudaDriverEntryPointSuccess && fn) {
      g_encode_tiled = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
      g_encode_state = 1;
    } else {
      (void)cudaGetLastError();
      g_encode_state = 2;
    }
  }
  return g_encode_state == 1;
}

// A [B, T, M, width] BF16 tensor (element strides s0 batch, s1 time, s2 middle;
// innermost contiguous) as a 4-D map {width, M, T, B} with boxes of
// {min(width, 64), 1, 64, 1}: 64 consecutive time steps of one (batch, middle)
// row as [64][box width] in shared memory, 128-byte swizzled when the box is
// 128 bytes wide. Middle stride 0 (heads sharing the angles) is described as a
// middle dimension of extent 1.
bool encode_rows(CUtensorMap* map, const bf16* base, int width, int T, int M, int B, int64_t s0, int64_t s1,
                 int64_t s2) {
  if (s2 == 0) M = 1;
  const int64_t st2 = s2 == 0 ? width : s2;
  if (reinterpret_cast<uintptr_t>(base) % 16 || (st2 * 2) % 16 || (s1 * 2) % 16 || (s0 * 2) % 16) return false;
  const cuuint64_t dims[4] = {static_cast<cuuint64_t>(width), static_cast<cuuint64_t>(M), static_cast<cuuint64_t>(T),
                              static_cast<cuuint64_t>(B)};
  const cuuint64_t strides[3] = {static_cast<cuuint64_t>(st2 * 2), static_cast<cuuint64_t>(s1 * 2),
                                 static_cast<cuuint64_t>(s0 * 2)};
  const cuuint32_t box[4] = {static_cast<cuuint32_t>(width > 64 ? 64 : width), 1, kChunk, 1};
  const cuuint32_t elem[4] = {1, 1, 1, 1};
  const bool sw = width >= 64;
  return g_encode_tiled(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<bf16*>(base), dims, strides, box, elem,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, sw ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// Tensor maps of one direction; false (the launch then stages with cp.async) when a
// tensor's layout does not allow them.
bool encode_direction(RecurrenceParams& p) {
  if (!encode_available() || p.sa[3] != 1) return false;
  return encode_rows(&p.tm_q, p.q, kState, p.T, p.Hq, p.B, p.sq[0], p.sq[1], p.sq[2]) &&
         encode_rows(&p.tm_k, p.k, kState, p.T, p.Hq, p.B, p.sk[0], p.sk[1], p.sk[2]) &&
         encode_rows(&p.tm_v, p.v, kHead, p.T, p.H, p.B, p.sv[0], p.sv[1], p.sv[2]) &&
         encode_rows(&p.tm_z, p.z, kHead, p.T, p.H, p.B, p.sz[0], p.sz[1], p.sz[2]) &&
         encode_rows(&p.tm_a, p.ang, kRotary, p.T, p.H, p.B, p.sa[0], p.sa[1], p.sa[2]);
}

// Largest element offset + 1 of a tensor with these extents and (non-negative) strides.
int64_t extent(std::initializer_list<int64_t> dims, const int64_t* strides) {
  int64_t last = 0, i = 0;
  for (int64_t d : dims) {
    if (d <= 0) return 0;
    last += (d - 1) * strides[i++];
  }
  return last + 1;
}

void set_extents(RecurrenceParams& p) {
  p.ext_q = extent({p.B, p.T, p.Hq, kState}, p.sq);
  p.ext_k = extent({p.B, p.T, p.Hq, kState}, p.sk);
  p.ext_v = extent({p.B, p.T, p.H, kHead}, p.sv);
  p.ext_z = extent({p.B, p.T, p.H, kHead}, p.sz);
  p.ext_out = extent({p.B, p.T, p.H, kHead}, p.so);
  p.ext_a = extent({p.B, p.T, p.H, kRotary}, p.sa);
  p.ext_dt = extent({p.B, p.H, p.T}, p.sdt);
  p.ext_adt = extent({p.B, p.H, p.T}, p.sadt);
  p.ext_trap = extent({p.B, p.H, p.T}, p.str);
  p.ext_ar = p.raw_controls ? extent({p.B, p.T, p.H}, p.sar) : 0;
  p.ext_dr = p.raw_controls ? extent({p.B, p.T, p.H}, p.sdr) : 0;
}

int alignment_class(const RecurrenceLaunch& L) {
  int a = alignment_class_one(L.dir[0]);
  if (L.ndir > 1) a = a < alignment_class_one(L.dir[1]) ? a : alignment_class_one(L.dir[1]);
  return a;
}

template <int kVec, int kDirs, bool kExt, bool kTma = false>
int launch(const RecurrenceLaunch& L, unsigned char* ws, cudaStream_t stream) {
  const RecurrenceParams& p = L.dir[0];
  const int units = ((p.T + kChunk - 1) / kChunk) * p.B * p.H * L.ndir;
  const int grid = units < sm_count() ? units : sm_count();
  const bool look = (p.T + kChunk - 1) / kChunk > kLookbackChunks;
  if constexpr (kDirs == 2) {
    auto kernel = look ? recurrence_pair_kernel<kVec, true, kTma> : recurrence_pair_kernel<kVec, false, kTma>;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(L.dir[0], L.dir[1], ws);
  } else {
    auto kernel = look ? recurrence_persistent_kernel<kVec, kExt, true, kTma>
                       : recurrence_persistent_kernel<kVec, kExt, false, kTma>;
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(kSmemBytes));
    kernel<<<grid, kThreads, kSmemBytes, stream>>>(L.dir[0], ws);
  }
  return 0;
}

}  // namespace

size_t recurrence_workspace_bytes(int B, int T, int H, int ndir) {
  const size_t units = static_cast<size_t>((T + kChunk - 1) / kChunk) * B * H * ndir;
  return kWsHeader + units * kUnitBytes;
}

int launch_recurrence_persistent(const RecurrenceLaunch& launch_in, void* workspace, size_t workspace_bytes,
                                 cudaStream_t stream) {
  if (launch_in.ndir < 1 || launch_in.ndir > 2) return 1;
  RecurrenceLaunch L = launch_in;
  for (int i = 0; i < L.ndir; ++i) {
    L.dir[i].ang_vec = angles_vectorizable(L.dir[i]);
    L.dir[i].flag_wait_ns = flag_wait_limit_ns();
    L.dir[i].err_host = host_error_word();
    set_extents(L.dir[i]);
  }
  const RecurrenceParams& p = L.dir[0];
  if (workspace_bytes < recurrence_workspace_bytes(p.B, p.T, p.H, L.ndir)) return 1;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const int a = alignment_class(L);
  // TMA staging for 16-byte rows of long rows (more than kLookbackChunks chunks), when
  // every direction's tensors allow it: there it measured faster than per-thread
  // cp.async (137.3 against 138.2 us at B=2, T=3600); for short rows cp.async is
  // faster (41.8 against 43.7 us at B=16, T=200), where the first unit's rows are on
  // the launch's critical path.
  bool tma = a == 16 && (p.T + kChunk - 1) / kChunk > kLookbackChunks;
  for (int i = 0; i < L.ndir && tma; ++i) tma = encode_direction(L.dir[i]);
  for (int i = 0; i < L.ndir; ++i) L.dir[i].tma = tma ? 1 : 0;
  bool ext = false;
  for (int i = 0; i < L.ndir; ++i) ext = ext || L.dir[i].reverse || L.dir[i].raw_controls;
  if (tma)
    return L.ndir == 2 ? launch<16, 2, true, true>(L, ws, stream)
                       : ext ? launch<16, 1, true, true>(L, ws, stream) : launch<16, 1, false, true>(L, ws, stream);
  if (L.ndir == 2)
    return a == 16 ? launch<16, 2, true>(L, ws, stream)
                   : a == 8 ? launch<8, 2, true>(L, ws, stream) : launch<2, 2, true>(L, ws, stream);
  if (ext)
    return a == 16 ? launch<16, 1, true>(L, ws, stream)
                   : a == 8 ? launch<8, 1, true>(L, ws, stream) : launch<2, 1, true>(L, ws, stream);
  return a == 16 ? launch<16, 1, false>(L, ws, stream)
                 : a == 8 ? launch<8, 1, false>(L, ws, stream) : launch<2, 1, false>(L, ws, stream);
}

int read_device_error(int reset) {
  int v = 0;
  cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int));
  if (reset) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int));
    if (int* w = host_error_word()) *reinterpret_cast<volatile int*>(w) = 0;
  }
  return v;
}

}  // namespace tf

// ===================================================================================
// Entry point that allocates nothing.
//
// Some callers of this library cannot allocate device memory: plugin hosts that
// own all GPU memory through their own pool and give plugins no allocation hook,
// and latency-critical services that forbid cudaMalloc after start-up (it can
// synchronise the device and take milliseconds). They call
// tf_mamba_recurrence_fwd_static, whose workspace is the file-scope array below
// instead of a caller buffer.
//
// Limits and rules:
//   - The array holds kStaticWorkspaceBytes (64 MiB). Every GPU that loads this
//     library keeps that much device memory until the process exits. Problems
//     whose workspace (tf_recurrence_workspace_size) exceeds it are rejected with
//     TF_ERR_SIZE before anything is launched.
//   - The first call on a device looks up the array's device address there
//     (cudaGetSymbolAddress, with that device current) and caches it; make that
//     first call before any stream capture. With CUDA's lazy module loading the
//     array is reserved when this file's module first loads on the device, which
//     can be that first call: make it at start-up, before a memory pool takes the
//     device's memory. If the array cannot be had, the call returns
//     TF_ERR_DEVICE and tf_last_cuda_error names the cause.
//   - All calls on a device share the one array. Each call first clears what
//     the kernel needs at zero (the workspace header and every chunk flag), so
//     a call never depends on what an earlier call left behind, but calls that
//     overlap on the GPU race with each other: serialise them.
// ===================================================================================
namespace tf {
namespace {

constexpr size_t kStaticWorkspaceBytes = size_t{64} << 20;
__device__ __align__(256) unsigned char g_static_workspace[kStaticWorkspaceBytes];

void* g_static_ptr[kMaxDevices] = {nullptr};

// Device address of g_static_workspace on the current device (set up once).
// TF_OK, or TF_ERR_DEVICE with the cause recorded.
int static_workspace(void** out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    snprintf(g_last_error, sizeof g_last_error, "no usable current CUDA device");
    return TF_ERR_DEVICE;
  }
  if (g_static_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_static_workspace);
    if (e != cudaSuccess || ptr == nullptr) {
      // With lazy module loading this is where the module (and the array) is first
      // loaded on the device; it fails when no device memory is left for it.
      snprintf(g_last_error, sizeof g_last_error, "static workspace unavailable on device %d: %s", dev,
               cudaGetErrorString(e));
      (void)cudaGetLastError();
      return TF_ERR_DEVICE;
    }
    g_static_ptr[dev] = ptr;
  }
  *out = g_static_ptr[dev];
  return TF_OK;
}

}  // namespace

// Clears the static workspace's header and chunk flags on `stream`, then
// returns its address and capacity. TF_OK, or an error status with the cause
// recorded.
int prepare_static_workspace(int B, int T, int H, cudaStream_t stream, void** ws, size_t* bytes) {
  void* ptr = nullptr;
  const int st = static_workspace(&ptr);
  if (st != TF_OK) return st;
  const size_t units = static_cast<size_t>((T + kChunk - 1) / kChunk) * B * H;
  unsigned char* base = static_cast<unsigned char*>(ptr);
  cudaError_t e = cudaMemsetAsync(base, 0, kWsHeader, stream);
  if (e == cudaSuccess && units > 0)
    e = cudaMemset2DAsync(base + kWsHeader + kUnitFlag, kUnitBytes, 0, sizeof(uint32_t), units, stream);
  if (e != cudaSuccess) {
    snprintf(g_last_error, sizeof g_last_error, "%s", cudaGetErrorString(e));
    return TF_ERR_LAUNCH;
  }
  *ws = ptr;
  *bytes = kStaticWorkspaceBytes;
  return TF_OK;
}

size_t static_workspace_capacity() { return kStaticWorkspaceBytes; }

}  // namespace tf
