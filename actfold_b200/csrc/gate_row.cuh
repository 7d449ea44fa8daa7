// Per-row similarity device functions shared by the dense gate (af_gate) and
// the packed-row gate inside the native folded pass.
#pragma once

#include "common.cuh"

namespace af {

struct GateConsts {
  float tau_r;     // tau rounded to the input dtype
  float eps_r;     // eps rounded to the input dtype (cosine norm clamp)
  float eps;       // eps as f32 (pearson denominator)
  float l2_denom;  // sqrt(H) + eps evaluated in double, as f32
};

struct GateOut {
  uint8_t stable;
  float sim;
  float ss_c = -1.f;  // cosine metric: the candidate row's reduced fp32 sum of squares (else -1)
};

// Host-side rounding to a storage dtype (round to nearest even).
inline float host_round(float x, int dtype) {
  if (dtype == AF_DTYPE_BF16) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return x;  // NaN
    u = (u + (((u >> 16) & 1u) + 0x7fffu)) & 0xffff0000u;
    float r;
    memcpy(&r, &u, 4);
    return r;
  }
  if (dtype == AF_DTYPE_F16) return __half2float(__float2half_rn(x));
  return x;
}

inline GateConsts make_gate_consts(int dtype, float tau, float eps, float l2_denom) {
  GateConsts k;
  k.tau_r = host_round(tau, dtype);
  k.eps_r = host_round(eps, dtype);
  k.eps = eps;
  k.l2_denom = l2_denom;
  return k;
}

// rnd<DT>(fp32(x / n)) with n already rounded; r = 1 / n (correctly rounded).
template <int DT>
__device__ __forceinline__ float quot(float x, float n, float r) {
  if constexpr (DT == AF_DTYPE_BF16) {
    float y = __fmul_rn(x, r);
    const int low = (int)(__float_as_uint(y) & 0xffffu) - 0x8000;
    if (low >= -4 && low <= 4) y = __fdiv_rn(x, n);  // near a bf16 midpoint: exact quotient
    return rnd<DT>(y);
  } else {
    return rnd<DT>(__fdiv_rn(x, n));
  }
}

template <int DT, int METRIC>
__device__ __forceinline__ float finish_cos(float sc, float sp, const GateConsts& k, float& nc, float& np) {
  nc = rnd<DT>(__fsqrt_rn(sc));
  np = rnd<DT>(__fsqrt_rn(sp));
  nc = nc < k.eps_r ? k.eps_r : nc;  // clamp_min keeps NaN
  np = np < k.eps_r ? k.eps_r : np;
  return 0.f;
}

// Threads that share one row and how they sum across it.
// WarpRows: one warp per row (the reduction is a shuffle tree).
struct WarpRows {
  static constexpr int kThreads = 32;
  __device__ __forceinline__ float sum(float v) const { return warp_sum(v); }
  __device__ __forceinline__ void sum2(float& a, float& b) const {
    a = warp_sum(a);
    b = warp_sum(b);
  }
};

// CtaRows<NT>: one CTA of NT threads per row. Warp partials go through
// `red` (2 * NT / 32 floats of shared memory) and every thread adds them in
// the same fixed order, so all threads hold the same total. Every thread of
// the CTA must call each reduction (they contain __syncthreads).
template <int NT>
struct CtaRows {
  static constexpr int kThreads = NT;
  float* red;
  __device__ __forceinline__ void sum2(float& a, float& b) const {
    a = warp_sum(a);
    b = warp_sum(b);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) {
      red[2 * w] = a;
      red[2 * w + 1] = b;
    }
    __syncthreads();
    float x = 0.f, y = 0.f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) {
      x += red[2 * i];
      y += red[2 * i + 1];
    }
    __syncthreads();
    a = x;
    b = y;
  }
  // One value: the same warp sums and the same order of the cross-warp adds
  // as sum2's first value, with half its shuffles and shared-memory reads.
  __device__ __forceinline__ float sum(float v) const {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float x = 0.f;
#pragma unroll
    for (int i = 0; i < NT / 32; ++i) x += red[i];
    __syncthreads();
    return x;
  }
};

// Row held in registers: thread `tid` of a G-thread row group owns vectors
// v = i * G + tid (zero past nvec).
template <int NV, int G = 32>
__device__ __forceinline__ void load_row(const char* p, int nvec, int tid, uint4 (&v)[NV]) {
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int j = i * G + tid;
    v[i] = j < nvec ? ldg16(p + 16 * (int64_t)j) : make_uint4(0u, 0u, 0u, 0u);
  }
}

template <int DT, int METRIC, int NV, class Rows = WarpRows>
__device__ __forceinline__ GateOut gate_regs(const uint4 (&cv)[NV], const uint4 (&pv)[NV], int nvec, int H,
                                             const GateConsts& k, int tid, const Rows& rows = Rows());

template <int DT, int METRIC, int NV>
__device__ __forceinline__ GateOut gate_row_vec(const char* c, const char* q, int nvec, int H, const GateConsts& k,
                                                int lane) {
  uint4 cv[NV], pv[NV];
  load_row<NV>(c, nvec, lane, cv);
  load_row<NV>(q, nvec, lane, pv);
  return gate_regs<DT, METRIC, NV>(cv, pv, nvec, H, k, lane);
}

template <int DT, int METRIC, int NV, class Rows>
__device__ __forceinline__ GateOut gate_regs(const uint4 (&cv)[NV], const uint4 (&pv)[NV], int nvec, int H,
                                             const GateConsts& k, int tid, const Rows& rows) {
  constexpr int E = Elt<DT>::kPerVec;
  constexpr int G = Rows::kThreads;
  float presum;
  float ss_c = -1.f;
  if constexpr (METRIC == AF_METRIC_COSINE) {
    float sc = 0.f, sp = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float fc[E], fp[E];
      unpack<DT>(cv[i], fc);
      unpack<DT>(pv[i], fp);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        sc = fmaf(fc[e], fc[e], sc);
        sp = fmaf(fp[e], fp[e], sp);
      }
    }
    rows.sum2(sc, sp);
    ss_c = sc;
    float nc, np;
    finish_cos<DT, METRIC>(sc, sp, k, nc, np);
    const float rc = __frcp_rn(nc), rp = __frcp_rn(np);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (i * G + tid >= nvec) continue;
      float fc[E], fp[E];
      unpack<DT>(cv[i], fc);
      unpack<DT>(pv[i], fp);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float yc = quot<DT>(fc[e], nc, rc);
        const float yp = quot<DT>(fp[e], np, rp);
        s = __fadd_rn(s, rnd<DT>(__fmul_rn(yc, yp)));
      }
    }
    presum = rows.sum(s);
  } else if constexpr (METRIC == AF_METRIC_L2) {
    float sd = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (i * G + tid >= nvec) continue;
      float fc[E], fp[E];
      unpack<DT>(cv[i], fc);
      unpack<DT>(pv[i], fp);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float d = rnd<DT>(__fsub_rn(fc[e], fp[e]));
        sd = fmaf(d, d, sd);
      }
    }
    sd = rows.sum(sd);
    const float l2 = rnd<DT>(__fsqrt_rn(sd));
    presum = __fsub_rn(1.f, rnd<DT>(__fdiv_rn(l2, k.l2_denom)));
  } else {  // pearson
    float mc = 0.f, mp = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (i * G + tid >= nvec) continue;
      float fc[E], fp[E];
      unpack<DT>(cv[i], fc);
      unpack<DT>(pv[i], fp);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        mc = __fadd_rn(mc, fc[e]);
        mp = __fadd_rn(mp, fp[e]);
      }
    }
    rows.sum2(mc, mp);
    mc = rnd<DT>(__fdiv_rn(mc, (float)H));
    mp = rnd<DT>(__fdiv_rn(mp, (float)H));
    float num = 0.f, scc = 0.f, spp = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      if (i * G + tid >= nvec) continue;
      float fc[E], fp[E];
      unpack<DT>(cv[i], fc);
      unpack<DT>(pv[i], fp);
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float cc = rnd<DT>(__fsub_rn(fc[e], mc));
        const float pc = rnd<DT>(__fsub_rn(fp[e], mp));
        num = __fadd_rn(num, rnd<DT>(__fmul_rn(cc, pc)));
        scc = fmaf(cc, cc, scc);
        spp = fmaf(pc, pc, spp);
      }
    }
    rows.sum2(num, scc);
    spp = rows.sum(spp);
    const float numr = rnd<DT>(num);
    const float nc = rnd<DT>(__fsqrt_rn(scc));
    const float np = rnd<DT>(__fsqrt_rn(spp));
    const float den = rnd<DT>(__fadd_rn(rnd<DT>(__fmul_rn(nc, np)), k.eps));
    presum = __fdiv_rn(numr, den);
  }
  GateOut o;
  o.sim = rnd<DT>(presum);
  o.stable = o.sim > k.tau_r ? 1 : 0;
  o.ss_c = ss_c;
  return o;
}

// bf16 x / n for bf16 x and n > 0: x * (1/n) in fp32 rounds to the same bf16
// value as the fp32 quotient. The exact quotient of two bf16 values is never a
// bf16 rounding midpoint (a midpoint has an odd 9-bit significand M, and
// x = M * n / 2^s would need 2^s to divide n's 8-bit significand, leaving
// x's significand >= M > 255), and when it is not one it lies at least 2^-17
// (relative) away from every midpoint, while the product and the quotient are
// within 2^-23 of it. Only results in the subnormal range, where those bounds
// do not hold, take the IEEE division.
__device__ __forceinline__ float quot_bf16(float x, float n, float r) {
  float y = __fmul_rn(x, r);
  if (fabsf(y) < 0x1p-125f) y = __fdiv_rn(x, n);
  return y;  // rounded to bf16 by the caller
}

// Packed pair arithmetic (sm_100): two fp32 lanes in one 64-bit register
// (element 0 in the low half) and bf16x2 words (element 0 in the low half).
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// bf16x2 word of rnd(lo), rnd(hi) (round to nearest even).
__device__ __forceinline__ uint32_t bf2_round(uint64_t v) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(f2_hi(v)), "f"(f2_lo(v)));
  return r;
}
// Both products of two bf16x2 words, each rounded once to bf16.
__device__ __forceinline__ uint32_t bf2_mul(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// A bf16x2 word as two fp32 lanes (exact).
__device__ __forceinline__ uint64_t bf2_widen(uint32_t w) { return f2_pack(bf16_lo(w), bf16_hi(w)); }

// rnd_bf16(sqrt(x)) for x >= 0: the approximate square root (within a few
// fp32 ulp), and the IEEE one only where the approximation lies within 8 ulp
// of a bf16 rounding midpoint, so the bf16 result is that of the exact root.
__device__ __forceinline__ float sqrt_to_bf16(float x) {
  float s;
  asm("sqrt.approx.f32 %0, %1;" : "=f"(s) : "f"(x));
  const int low = (int)(__float_as_uint(s) & 0xffffu) - 0x8000;
  if (low >= -8 && low <= 8) s = __fsqrt_rn(x);
  return rnd<AF_DTYPE_BF16>(s);
}

// 1 / n for a bf16 n > 0, for the quotients x * (1/n) of bf16 values: the
// approximate reciprocal is within 2^-22 of 1/n, and every exact quotient of
// two bf16 values that is not an fp32 subnormal lies at least 2^-17 (relative)
// from a bf16 rounding midpoint (quot_bf16), so x * (1/n) still rounds to the
// bf16 value of x / n.
__device__ __forceinline__ float rcp_for_bf16_quot(float n) {
  float r;
  asm("rcp.approx.f32 %0, %1;" : "=f"(r) : "f"(n));
  return r;
}

// gate_regs<bf16, cosine> with the same per-thread order of every fp32 sum, so
// the same similarity bit for bit, in fewer instructions: the row's floats are
// kept from the norm pass, the normalised values and their products are
// rounded two at a time (cvt.rn.bf16x2.f32), and the quotient needs no check
// (quot_bf16). The product of two bf16 values is exact in fp32, so rounding it
// once equals rnd(fmul).
template <int NV, class Rows>
__device__ __forceinline__ GateOut gate_regs_bf16_cos(const uint4 (&cv)[NV], const uint4 (&pv)[NV], int nvec,
                                                      const GateConsts& k, int tid, const Rows& rows) {
  constexpr int G = Rows::kThreads;
  float fc[NV][8], fp[NV][8];
  float sc = 0.f, sp = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    unpack<AF_DTYPE_BF16>(cv[i], fc[i]);
    unpack<AF_DTYPE_BF16>(pv[i], fp[i]);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      sc = fmaf(fc[i][e], fc[i][e], sc);
      sp = fmaf(fp[i][e], fp[i][e], sp);
    }
  }
  rows.sum2(sc, sp);
  float nc, np;
  finish_cos<AF_DTYPE_BF16, AF_METRIC_COSINE>(sc, sp, k, nc, np);
  const float rc = __frcp_rn(nc), rp = __frcp_rn(np);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    if (i * G + tid >= nvec) continue;
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float2 yc = __bfloat1622float2(
          __floats2bfloat162_rn(quot_bf16(fc[i][e], nc, rc), quot_bf16(fc[i][e + 1], nc, rc)));
      const float2 yp = __bfloat1622float2(
          __floats2bfloat162_rn(quot_bf16(fp[i][e], np, rp), quot_bf16(fp[i][e + 1], np, rp)));
      const float2 pr = __bfloat1622float2(__floats2bfloat162_rn(__fmul_rn(yc.x, yp.x), __fmul_rn(yc.y, yp.y)));
      s = __fadd_rn(s, pr.x);
      s = __fadd_rn(s, pr.y);
    }
  }
  GateOut o;
  o.sim = rnd<AF_DTYPE_BF16>(rows.sum(s));
  o.stable = o.sim > k.tau_r ? 1 : 0;
  o.ss_c = sc;
  return o;
}

// Scalar fallback: any H and alignment; re-reads the row for each pass.
template <int DT, int METRIC>
__device__ __forceinline__ GateOut gate_row_scalar(const char* c, const char* q, int H, const GateConsts& k,
                                                   int lane) {
  float presum;
  if constexpr (METRIC == AF_METRIC_COSINE) {
    float sc = 0.f, sp = 0.f;
    for (int i = lane; i < H; i += 32) {
      const float a = load_scalar<DT>(c, i), b = load_scalar<DT>(q, i);
      sc = fmaf(a, a, sc);
      sp = fmaf(b, b, sp);
    }
    sc = warp_sum(sc);
    sp = warp_sum(sp);
    float nc, np;
    finish_cos<DT, METRIC>(sc, sp, k, nc, np);
    const float rc = __frcp_rn(nc), rp = __frcp_rn(np);
    float s = 0.f;
    for (int i = lane; i < H; i += 32) {
      const float yc = quot<DT>(load_scalar<DT>(c, i), nc, rc);
      const float yp = quot<DT>(load_scalar<DT>(q, i), np, rp);
      s = __fadd_rn(s, rnd<DT>(__fmul_rn(yc, yp)));
    }
    presum = warp_sum(s);
  } else if constexpr (METRIC == AF_METRIC_L2) {
    float sd = 0.f;
    for (int i = lane; i < H; i += 32) {
      const float d = rnd<DT>(__fsub_rn(load_scalar<DT>(c, i), load_scalar<DT>(q, i)));
      sd = fmaf(d, d, sd);
    }
    const float l2 = rnd<DT>(__fsqrt_rn(warp_sum(sd)));
    presum = __fsub_rn(1.f, rnd<DT>(__fdiv_rn(l2, k.l2_denom)));
  } else {
    float mc = 0.f, mp = 0.f;
    for (int i = lane; i < H; i += 32) {
      mc = __fadd_rn(mc, load_scalar<DT>(c, i));
      mp = __fadd_rn(mp, load_scalar<DT>(q, i));
    }
    mc = rnd<DT>(__fdiv_rn(warp_sum(mc), (float)H));
    mp = rnd<DT>(__fdiv_rn(warp_sum(mp), (float)H));
    float num = 0.f, scc = 0.f, spp = 0.f;
    for (int i = lane; i < H; i += 32) {
      const float cc = rnd<DT>(__fsub_rn(load_scalar<DT>(c, i), mc));
      const float pc = rnd<DT>(__fsub_rn(load_scalar<DT>(q, i), mp));
      num = __fadd_rn(num, rnd<DT>(__fmul_rn(cc, pc)));
      scc = fmaf(cc, cc, scc);
      spp = fmaf(pc, pc, spp);
    }
    const float numr = rnd<DT>(warp_sum(num));
    const float nc = rnd<DT>(__fsqrt_rn(warp_sum(scc)));
    const float np = rnd<DT>(__fsqrt_rn(warp_sum(spp)));
    const float den = rnd<DT>(__fadd_rn(rnd<DT>(__fmul_rn(nc, np)), k.eps));
    presum = __fdiv_rn(numr, den);
  }
  GateOut o;
  o.sim = rnd<DT>(presum);
  o.stable = o.sim > k.tau_r ? 1 : 0;
  return o;
}

}  // namespace af
