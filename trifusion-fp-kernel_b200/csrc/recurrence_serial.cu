// Fused Mamba-3 SISO recurrence, serial-chunk form: one CTA per (batch, head)
// walks the sequence in 64-step chunks, carrying the 64x128 FP32 state in the
// registers of its four warps. This is the arithmetic of the reference kernel
// `_fused` (mamba_fused.py:72-152), restated for CUDA:
//
//   controls  gamma = dt*sigmoid(trap), scale = dt[t+1]*(1-sigmoid(trap[t+1])) + gamma   (:96-101)
//   angles    phase = (cumsum tanh(raw)*pi*dt + carry) mod 2pi, first 32 pairs     (:102-111)
//   q/k       q += qb, k += kb; qk = sum(q*k)*gamma; qr = rot(q); kr = rot(k)*scale (:112-135)
//   decay     da = adt*log2 e, cs = cumsum(da), total = sum(da)                     (:140-142)
//   output    acc = (qr S^T) 2^cs + tril(qr kr^T 2^min(cs_i-cs_j,0)) v + (D+qk) v;
//             out = acc * z*sigmoid(z)                                               (:143-149)
//   state     S = S 2^total + v^T (kr 2^(total-cs))                                  (:151-152)
//
// Precision. The reference rounds qr, kr, the state, the decayed scores and the
// decay-weighted v to BF16 before its dot products; on the benchmark
// distributions that alone puts it 2.3e-3 (relative L2) from its own FP32 path.
// Here every tensor-core operand is FP16 (3 more mantissa bits) with a
// per-row power-of-two exponent that keeps it inside FP16's range; the decayed
// scores are split into FP16 hi + lo halves (two MMAs); the decay weight of the
// state update multiplies kr instead of v, so v enters the MMA unrounded. All
// accumulation is FP32. The result stays within 1e-2 (abs) + 1e-2 (rel) of the
// reference's FP32 path.
#include "recurrence.cuh"

namespace tf {
namespace {

constexpr int kThreads = 128;
constexpr int kNP = kState + 8;  // padded 16-bit row of a 128-wide tile (conflict-free ldmatrix)
constexpr int kPP = kHead + 8;   // padded 16-bit row of a 64-wide tile

struct SerialSmem {
  __half q[kChunk][kNP];    // fp16(qr_i * 2^qe_i)
  __half k[kChunk][kNP];    // fp16(kr_j * 2^ke_j)
  __half kw[kChunk][kNP];   // fp16(kr_j * 2^(total - cs_j))
  __half s[kHead][kNP];     // fp16(S[p] * 2^se_p)
  bf16 v[kChunk][kPP];      // v as loaded (skip term)
  __half v16[kChunk][kPP];  // v as an FP16 MMA operand
  bf16 z[kChunk][kPP];      // z in; output staging out (same positions)
  float phase[kChunk][kRotary + 1];
  float seg[4][kRotary];    // per-warp partial angle sums
  float carry[kRotary];     // angle carry, mod 2pi
  float dtc[kChunk];
  float gamma[kChunk];
  float scale[kChunk];
  float cs[kChunk];
  float qk[kChunk];
  float qe[kChunk];         // row exponents of the FP16 q tile (as floats)
  float ke[kChunk];         // row exponents of the FP16 k tile
  float sinv[kHead];        // 2^-se_p
  float wsum[2];
};

template <bool kAligned>
struct Loader {
  // Two consecutive BF16 elements (innermost stride 1) as floats.
  static __device__ __forceinline__ float2 pair(const bf16* p) {
    if constexpr (kAligned) {
      return unpack_bf16x2(*reinterpret_cast<const uint32_t*>(p));
    } else {
      return make_float2(bf2f(p[0]), bf2f(p[1]));
    }
  }
};

__device__ __forceinline__ float load_trap(const RecurrenceParams& p, const void* base, int64_t off) {
  return p.trap_bf16 ? bf2f(static_cast<const bf16*>(base)[off])
                     : static_cast<const float*>(base)[off];
}

// Maximum over the 4 lanes of an MMA quad (lanes sharing one fragment row).
__device__ __forceinline__ float quad_max(float x) {
  x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 1));
  return fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 2));
}

template <bool kAligned>
__global__ void __launch_bounds__(kThreads, 2) recurrence_serial_kernel(RecurrenceParams p) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  SerialSmem& sm = *reinterpret_cast<SerialSmem*>(smem_raw);
  using L = Loader<kAligned>;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, c4 = lane & 3;
  const int b = blockIdx.x / p.H, h = blockIdx.x % p.H;
  const int qh = h / (p.H / p.Hq);
  int T_eff = p.T;
  if (p.lengths) {
    const int64_t len = p.lengths[b];
    T_eff = static_cast<int>(len < 0 ? 0 : (len > p.T ? p.T : len));
  }

  const bf16* qbase = p.q + b * p.sq[0] + qh * p.sq[2];
  const bf16* kbase = p.k + b * p.sk[0] + qh * p.sk[2];
  const bf16* vbase = p.v + b * p.sv[0] + h * p.sv[2];
  const bf16* zbase = p.z + b * p.sz[0] + h * p.sz[2];
  const bf16* abase = p.ang + b * p.sa[0] + h * p.sa[2];
  bf16* obase = p.out + b * p.so[0] + h * p.so[2];
  const float* dtbase = p.dt + b * p.sdt[0] + h * p.sdt[1];
  const float* adtbase = p.adt + b * p.sadt[0] + h * p.sadt[1];
  const char* trbase = static_cast<const char*>(p.trap) +
                       (b * p.str[0] + h * p.str[1]) * (p.trap_bf16 ? 2 : 4);
  const float skip = p.d[h];

  // Per-lane constants for the 4 q/k columns this lane owns.
  const int col0 = 4 * lane;
  float qbias[4], kbias[4], qwv[4], kwv[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    qbias[e] = p.qb[h * kState + col0 + e];
    kbias[e] = p.kb[h * kState + col0 + e];
    qwv[e] = p.qw ? p.qw[col0 + e] : 1.f;
    kwv[e] = p.kw ? p.kw[col0 + e] : 1.f;
  }

  // State rows p = 16*warp .. 16*warp+15 live in this warp's registers:
  // S[nb][*] is the m16n8 accumulator block for state columns 8*nb .. 8*nb+7.
  float S[16][4];
#pragma unroll
  for (int nb = 0; nb < 16; ++nb) S[nb][0] = S[nb][1] = S[nb][2] = S[nb][3] = 0.f;
  for (int i = tid; i < kHead * kNP; i += kThreads) (&sm.s[0][0])[i] = __float2half_rn(0.f);
  if (tid < kHead) sm.sinv[tid] = 1.f;
  if (tid < kRotary) sm.carry[tid] = 0.f;

  for (int c0 = 0; c0 < T_eff; c0 += kChunk) {
    __syncthreads();
    // ---- A. controls and the decay cumsum (threads 0..63, one step each) ----
    if (tid < kChunk) {
      const int pos = c0 + tid;
      const bool valid = pos < T_eff;
      const bool next = pos + 1 < T_eff;
      const float dtv = valid ? dtbase[pos * p.sdt[2]] : 0.f;
      const float dn = next ? dtbase[(pos + 1) * p.sdt[2]] : 0.f;
      const float trv = sigmoidf_fast(valid ? load_trap(p, trbase, pos * p.str[2]) : 0.f);
      const float tnv = sigmoidf_fast(next ? load_trap(p, trbase, (pos + 1) * p.str[2]) : 0.f);
      const float gm = dtv * trv;
      float x = valid ? adtbase[pos * p.sadt[2]] * kLog2e : 0.f;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane == 31) sm.wsum[warp] = x;
      sm.dtc[tid] = dtv;
      sm.gamma[tid] = gm;
      sm.scale[tid] = dn * (1.f - tnv) + gm;
      sm.cs[tid] = x;
    }
    __syncthreads();
    if (tid >= 32 && tid < kChunk) sm.cs[tid] += sm.wsum[0];
    // ---- B. angle partial cumsums: lane = pair r, warp = 16-step segment ----
    {
      const int r = lane, t0 = warp * 16;
      float run = 0.f;
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int t = t0 + i, pos = c0 + t;
        const float raw = pos < T_eff ? bf2f(abase[pos * p.sa[1] + r * p.sa[3]]) : 0.f;
        run += (tanh_approx(raw) * kPi) * sm.dtc[t];
        sm.phase[t][r] = run;
      }
      sm.seg[warp][r] = run;
    }
    __syncthreads();
    {
      const int r = lane, t0 = warp * 16;
      float off = sm.carry[r];
      for (int s = 0; s < warp; ++s) off += sm.seg[s][r];
#pragma unroll 4
      for (int i = 0; i < 16; ++i) {
        const int t = t0 + i;
        const float ph = sm.phase[t][r] + off;
        sm.phase[t][r] = ph - kTwoPi * floorf(ph / kTwoPi);
      }
    }
    __syncthreads();
    if (tid < kRotary) {
      const float c = sm.carry[tid] + ((sm.seg[0][tid] + sm.seg[1][tid]) + (sm.seg[2][tid] + sm.seg[3][tid]));
      sm.carry[tid] = c - kTwoPi * floorf(c / kTwoPi);
    }
    const float total = sm.cs[kChunk - 1];
    // ---- C. q/k rows: norm, bias, dot, rotation, scaling; v, z -------------
    for (int i = 0; i < 16; ++i) {
      const int t = warp * 16 + i, pos = c0 + t;
      uint2 qst = make_uint2(0, 0), kst = make_uint2(0, 0), kwst = make_uint2(0, 0);
      float qkv = 0.f;
      int qe = 0, ke = 0;
      if (pos < T_eff) {
        const bf16* qrow = qbase + pos * p.sq[1] + col0;
        const bf16* krow = kbase + pos * p.sk[1] + col0;
        const float2 q01 = L::pair(qrow), q23 = L::pair(qrow + 2);
        const float2 k01 = L::pair(krow), k23 = L::pair(krow + 2);
        float qv[4] = {q01.x, q01.y, q23.x, q23.y};
        float kv[4] = {k01.x, k01.y, k23.x, k23.y};
        if (p.qw) {  // C_norm: FP32 statistics, BF16 result (native.py:8-39)
          const float ss = warp_sum(qv[0] * qv[0] + qv[1] * qv[1] + qv[2] * qv[2] + qv[3] * qv[3]);
          const float rr = rsqrtf(ss / kState + p.eps);
#pragma unroll
          for (int e = 0; e < 4; ++e) qv[e] = bf16_round((qv[e] * rr) * qwv[e]);
        }
        if (p.kw) {  // B_norm
          const float ss = warp_sum(kv[0] * kv[0] + kv[1] * kv[1] + kv[2] * kv[2] + kv[3] * kv[3]);
          const float rr = rsqrtf(ss / kState + p.eps);
#pragma unroll
          for (int e = 0; e < 4; ++e) kv[e] = bf16_round((kv[e] * rr) * kwv[e]);
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          qv[e] += qbias[e];
          kv[e] += kbias[e];
        }
        qkv = warp_sum(qv[0] * kv[0] + qv[1] * kv[1] + qv[2] * kv[2] + qv[3] * kv[3]);
        const float sc = sm.scale[t];
        float qr[4], kr[4];
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int pr = 2 * lane + e;  // rotation pair index
          float cn = 1.f, sn = 0.f;
          if (pr < kRotary) __sincosf(sm.phase[t][pr], &sn, &cn);
          const float a0 = qv[2 * e], a1 = qv[2 * e + 1];
          const float b0 = kv[2 * e], b1 = kv[2 * e + 1];
          qr[2 * e] = a0 * cn - a1 * sn;
          qr[2 * e + 1] = a0 * sn + a1 * cn;
          kr[2 * e] = (b0 * cn - b1 * sn) * sc;
          kr[2 * e + 1] = (b0 * sn + b1 * cn) * sc;
        }
        qe = pow2_scale_exponent(warp_max(fmaxf(fmaxf(fabsf(qr[0]), fabsf(qr[1])), fmaxf(fabsf(qr[2]), fabsf(qr[3])))));
        ke = pow2_scale_exponent(warp_max(fmaxf(fmaxf(fabsf(kr[0]), fabsf(kr[1])), fmaxf(fabsf(kr[2]), fabsf(kr[3])))));
        const float qs = exp2i(qe), ks = exp2i(ke), w = ex2_approx(total - sm.cs[t]);
        qst = make_uint2(pack_f16x2(qr[0] * qs, qr[1] * qs), pack_f16x2(qr[2] * qs, qr[3] * qs));
        kst = make_uint2(pack_f16x2(kr[0] * ks, kr[1] * ks), pack_f16x2(kr[2] * ks, kr[3] * ks));
        kwst = make_uint2(pack_f16x2(kr[0] * w, kr[1] * w), pack_f16x2(kr[2] * w, kr[3] * w));
      }
      *reinterpret_cast<uint2*>(&sm.q[t][col0]) = qst;
      *reinterpret_cast<uint2*>(&sm.k[t][col0]) = kst;
      *reinterpret_cast<uint2*>(&sm.kw[t][col0]) = kwst;
      if (lane == 0) {
        sm.qk[t] = qkv * sm.gamma[t];
        sm.qe[t] = static_cast<float>(qe);
        sm.ke[t] = static_cast<float>(ke);
      }
      // v, z: lane owns head columns 2*lane, 2*lane+1
      uint32_t vst = 0, v16st = 0, zst = 0;
      if (pos < T_eff) {
        const float2 vv = L::pair(vbase + pos * p.sv[1] + 2 * lane);
        const float2 zz = L::pair(zbase + pos * p.sz[1] + 2 * lane);
        vst = pack_bf16x2(vv.x, vv.y);
        v16st = pack_f16x2(vv.x, vv.y);
        zst = pack_bf16x2(zz.x, zz.y);
      }
      *reinterpret_cast<uint32_t*>(&sm.v[t][2 * lane]) = vst;
      *reinterpret_cast<uint32_t*>(&sm.v16[t][2 * lane]) = v16st;
      *reinterpret_cast<uint32_t*>(&sm.z[t][2 * lane]) = zst;
    }
    __syncthreads();

    // ---- D. output rows 16*warp .. 16*warp+15 --------------------------------
    const int m0 = warp * 16;
    float acc[8][4];
    float sc[8][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) acc[nb][e] = sc[nb][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < kState / 16; ++kk) {
      uint32_t a[4];
      ldsm_x4(a, &sm.q[m0 + (lane & 7) + ((lane >> 3) & 1) * 8][kk * 16 + (lane >> 4) * 8]);
#pragma unroll
      for (int nb2 = 0; nb2 < 4; ++nb2) {
        uint32_t bs[4], bk[4];
        // B = S^T: rows of the stored state are the n index (head column p).
        ldsm_x4(bs, &sm.s[nb2 * 16 + (lane & 7) + (lane >> 4) * 8][kk * 16 + ((lane >> 3) & 1) * 8]);
        mma_f16_16816(acc[2 * nb2], a, bs[0], bs[1]);
        mma_f16_16816(acc[2 * nb2 + 1], a, bs[2], bs[3]);
        // B = kr^T: rows of the stored kr are the n index (time step j).
        ldsm_x4(bk, &sm.k[nb2 * 16 + (lane & 7) + (lane >> 4) * 8][kk * 16 + ((lane >> 3) & 1) * 8]);
        mma_f16_16816(sc[2 * nb2], a, bk[0], bk[1]);
        mma_f16_16816(sc[2 * nb2 + 1], a, bk[2], bk[3]);
      }
    }
    const int i0 = m0 + g, i1 = m0 + g + 8;
    const float cs0 = sm.cs[i0], cs1 = sm.cs[i1];
    const float qe0 = sm.qe[i0], qe1 = sm.qe[i1];
    // Inter-chunk term: undo the q row and state row exponents, apply 2^cs_i.
    const float r0 = ex2_approx(cs0 - qe0), r1 = ex2_approx(cs1 - qe1);
    float pmax0 = 0.f, pmax1 = 0.f;
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const int pc = nb * 8 + 2 * c4;
      const float s0 = sm.sinv[pc], s1 = sm.sinv[pc + 1];
      acc[nb][0] *= r0 * s0;
      acc[nb][1] *= r0 * s1;
      acc[nb][2] *= r1 * s0;
      acc[nb][3] *= r1 * s1;
      // Intra-chunk scores: causal mask, decay and the q/k row exponents in one ex2.
      const int j0 = pc;
      const float csj0 = sm.cs[j0], csj1 = sm.cs[j0 + 1];
      const float kej0 = sm.ke[j0], kej1 = sm.ke[j0 + 1];
      sc[nb][0] = i0 > j0 ? sc[nb][0] * ex2_approx(fminf(cs0 - csj0, 0.f) - qe0 - kej0) : 0.f;
      sc[nb][1] = i0 > j0 + 1 ? sc[nb][1] * ex2_approx(fminf(cs0 - csj1, 0.f) - qe0 - kej1) : 0.f;
      sc[nb][2] = i1 > j0 ? sc[nb][2] * ex2_approx(fminf(cs1 - csj0, 0.f) - qe1 - kej0) : 0.f;
      sc[nb][3] = i1 > j0 + 1 ? sc[nb][3] * ex2_approx(fminf(cs1 - csj1, 0.f) - qe1 - kej1) : 0.f;
      pmax0 = fmaxf(pmax0, fmaxf(fabsf(sc[nb][0]), fabsf(sc[nb][1])));
      pmax1 = fmaxf(pmax1, fmaxf(fabsf(sc[nb][2]), fabsf(sc[nb][3])));
    }
    // Decayed scores as FP16 hi + lo A fragments, each row scaled by 2^pe.
    const int pe0 = pow2_scale_exponent(quad_max(pmax0));
    const int pe1 = pow2_scale_exponent(quad_max(pmax1));
    const float ps0 = exp2i(pe0), ps1 = exp2i(pe1);
    uint32_t phi[4][4], plo[4][4];
#pragma unroll
    for (int nb = 0; nb < 8; ++nb) {
      const float a00 = sc[nb][0] * ps0, a01 = sc[nb][1] * ps0;
      const float a10 = sc[nb][2] * ps1, a11 = sc[nb][3] * ps1;
      const uint32_t h0 = pack_f16x2(a00, a01), h1 = pack_f16x2(a10, a11);
      const float2 f0 = unpack_f16x2(h0), f1 = unpack_f16x2(h1);
      phi[nb >> 1][(nb & 1) * 2 + 0] = h0;
      phi[nb >> 1][(nb & 1) * 2 + 1] = h1;
      plo[nb >> 1][(nb & 1) * 2 + 0] = pack_f16x2(a00 - f0.x, a01 - f0.y);
      plo[nb >> 1][(nb & 1) * 2 + 1] = pack_f16x2(a10 - f1.x, a11 - f1.y);
      acc[nb][0] *= ps0;
      acc[nb][1] *= ps0;
      acc[nb][2] *= ps1;
      acc[nb][3] *= ps1;
    }
#pragma unroll
    for (int kk = 0; kk < kChunk / 16; ++kk) {
#pragma unroll
      for (int nb2 = 0; nb2 < 4; ++nb2) {
        uint32_t bv[4];
        ldsm_x4_t(bv, &sm.v16[kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8][nb2 * 16 + (lane >> 4) * 8]);
        mma_f16_16816(acc[2 * nb2], phi[kk], bv[0], bv[1]);
        mma_f16_16816(acc[2 * nb2 + 1], phi[kk], bv[2], bv[3]);
        mma_f16_16816(acc[2 * nb2], plo[kk], bv[0], bv[1]);
        mma_f16_16816(acc[2 * nb2 + 1], plo[kk], bv[2], bv[3]);
      }
    }
    {
      const float u0 = exp2i(-pe0), u1 = exp2i(-pe1);
      const float sk0 = skip + sm.qk[i0], sk1 = skip + sm.qk[i1];
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        const int pc = nb * 8 + 2 * c4;
        const float2 v0 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.v[i0][pc]));
        const float2 v1 = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(&sm.v[i1][pc]));
        uint32_t* zp0 = reinterpret_cast<uint32_t*>(&sm.z[i0][pc]);
        uint32_t* zp1 = reinterpret_cast<uint32_t*>(&sm.z[i1][pc]);
        const float2 z0 = unpack_bf16x2(*zp0);
        const float2 z1 = unpack_bf16x2(*zp1);
        const float o00 = (acc[nb][0] * u0 + sk0 * v0.x) * (z0.x * sigmoidf_fast(z0.x));
        const float o01 = (acc[nb][1] * u0 + sk0 * v0.y) * (z0.y * sigmoidf_fast(z0.y));
        const float o10 = (acc[nb][2] * u1 + sk1 * v1.x) * (z1.x * sigmoidf_fast(z1.x));
        const float o11 = (acc[nb][3] * u1 + sk1 * v1.y) * (z1.y * sigmoidf_fast(z1.y));
        *zp0 = pack_bf16x2(o00, o01);  // z is consumed; its slot stages the output
        *zp1 = pack_bf16x2(o10, o11);
      }
    }
    __syncwarp();
    for (int i = 0; i < 16; ++i) {
      const int t = m0 + i, pos = c0 + t;
      if (pos < T_eff) {
        bf16* orow = obase + pos * p.so[1] + 2 * lane;
        const uint32_t val = *reinterpret_cast<const uint32_t*>(&sm.z[t][2 * lane]);
        if constexpr (kAligned) {
          *reinterpret_cast<uint32_t*>(orow) = val;
        } else {
          const float2 f = unpack_bf16x2(val);
          orow[0] = __float2bfloat16_rn(f.x);
          orow[1] = __float2bfloat16_rn(f.y);
        }
      }
    }
    __syncthreads();  // every warp has read sm.s / sm.sinv before they are rewritten

    // ---- E. state update for rows p = 16*warp .. +15 -------------------------
    const float gtot = ex2_approx(total);
#pragma unroll
    for (int nb = 0; nb < 16; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) S[nb][e] *= gtot;
#pragma unroll
    for (int kk = 0; kk < kChunk / 16; ++kk) {
      uint32_t a[4];
      // A[p][t] = v[t][p]: stored time-major, so load transposed.
      ldsm_x4_t(a, &sm.v16[kk * 16 + (lane & 7) + ((lane >> 4) & 1) * 8][m0 + ((lane >> 3) & 1) * 8]);
#pragma unroll
      for (int nb2 = 0; nb2 < 8; ++nb2) {
        uint32_t bk[4];
        ldsm_x4_t(bk, &sm.kw[kk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8][nb2 * 16 + (lane >> 4) * 8]);
        mma_f16_16816(S[2 * nb2], a, bk[0], bk[1]);
        mma_f16_16816(S[2 * nb2 + 1], a, bk[2], bk[3]);
      }
    }
    // FP16 copy of the state for the next chunk, each row p scaled by 2^se_p.
    float smax0 = 0.f, smax1 = 0.f;
#pragma unroll
    for (int nb = 0; nb < 16; ++nb) {
      smax0 = fmaxf(smax0, fmaxf(fabsf(S[nb][0]), fabsf(S[nb][1])));
      smax1 = fmaxf(smax1, fmaxf(fabsf(S[nb][2]), fabsf(S[nb][3])));
    }
    const int se0 = pow2_scale_exponent(quad_max(smax0));
    const int se1 = pow2_scale_exponent(quad_max(smax1));
    const float ss0 = exp2i(se0), ss1 = exp2i(se1);
#pragma unroll
    for (int nb = 0; nb < 16; ++nb) {
      const int n = nb * 8 + 2 * c4;
      *reinterpret_cast<uint32_t*>(&sm.s[m0 + g][n]) = pack_f16x2(S[nb][0] * ss0, S[nb][1] * ss0);
      *reinterpret_cast<uint32_t*>(&sm.s[m0 + g + 8][n]) = pack_f16x2(S[nb][2] * ss1, S[nb][3] * ss1);
    }
    if (c4 == 0) {
      sm.sinv[m0 + g] = exp2i(-se0);
      sm.sinv[m0 + g + 8] = exp2i(-se1);
    }
  }
  // Rows past the valid length are zero (length mask).
  if (T_eff < p.T) {
    for (int idx = tid; idx < (p.T - T_eff) * kHead; idx += kThreads) {
      const int t = T_eff + idx / kHead, c = idx % kHead;
      obase[t * p.so[1] + c] = __float2bfloat16_rn(0.f);
    }
  }
}

bool aligned4(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 3u) == 0; }

}  // namespace

int launch_recurrence_serial(const RecurrenceParams& p, cudaStream_t stream) {
  // The vectorised path reads BF16 pairs as 32-bit words: every BF16 tensor
  // needs 4-byte aligned rows (even strides, aligned base).
  bool al = aligned4(p.q) && aligned4(p.k) && aligned4(p.v) && aligned4(p.z) && aligned4(p.out);
  for (int i = 0; i < 3; ++i) {
    al = al && (p.sq[i] % 2 == 0) && (p.sk[i] % 2 == 0) && (p.sv[i] % 2 == 0) &&
         (p.sz[i] % 2 == 0) && (p.so[i] % 2 == 0);
  }
  const size_t smem = sizeof(SerialSmem);
  const dim3 grid(p.B * p.H), block(kThreads);
  if (al) {
    cudaFuncSetAttribute(recurrence_serial_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    recurrence_serial_kernel<true><<<grid, block, smem, stream>>>(p);
  } else {
    cudaFuncSetAttribute(recurrence_serial_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(smem));
    recurrence_serial_kernel<false><<<grid, block, smem, stream>>>(p);
  }
  return 0;
}

}  // namespace tf
