// Device-side arithmetic that reproduces the golden model's NumPy semantics.
//
// Rules (each mirrors a NumPy behaviour the golden simulator relies on):
//  * float32 arithmetic is IEEE round-to-nearest with no FMA contraction
//    (explicit __fmul_rn / __fadd_rn / __fdiv_rn / __fsqrt_rn);
//  * int32 -> float32 rounds to nearest (__int2float_rn);
//  * np.round is round-half-to-even (rintf);
//  * float32 -> float16 rounds to nearest even, overflow to inf;
//  * float64 -> float16 converts directly (cvt.rn.f16.f64), as np.float16(python float);
//  * float32 row sums follow NumPy's pairwise summation (8 accumulators per
//    leaf of <= 128 elements, halving split rounded to a multiple of 8) with
//    the additive identity as the initial value;
//  * mean / var divide in float64 and round to float32 (true_divide of a
//    float32 array by an intp count with out=float32);
//  * int8 casts of clipped values send NaN to 0; the int32 clip path sends
//    NaN and values >= 2^31 to INT32_MIN (x86 cvttss2si behaviour).
// exp, tanh and x**3 are evaluated in float64 and rounded once to float32;
// NumPy's own float32 SIMD versions are not correctly rounded, so these
// paths agree with the golden model to within one float32 ulp before the
// final FP16 rounding rather than bit-for-bit.
#pragma once
#include <cuda_fp16.h>
#include <cstdint>

namespace tac {

__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }
__device__ __forceinline__ uint16_t f2h(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ uint16_t d2h(double d) {
  uint16_t h;
  asm("cvt.rn.f16.f64 %0, %1;" : "=h"(h) : "d"(d));
  return h;
}

// np.clip(np.round(v), -128, 127).astype(np.int8) with NaN -> 0 (QUANT's rule and the
// REQUANT family's): one convert that rounds to nearest even, saturates to the int8
// range and turns NaN into 0 (PTX cvt.rni.sat.s8.f32, written to a 32-bit register).
__device__ __forceinline__ int8_t sat8(float v) {
  int32_t r;
  asm("cvt.rni.sat.s8.f32 %0, %1;" : "=r"(r) : "f"(v));
  return static_cast<int8_t>(r);
}

// np.clip(np.round(v), int32.min, int32.max).astype(np.int32) for float32 v
__device__ __forceinline__ int32_t sat32(float v) {
  float r = rintf(v);
  if (r != r || r >= 2147483648.f) return INT32_MIN;
  if (r <= -2147483648.f) return INT32_MIN;
  return static_cast<int32_t>(r);
}

__device__ __forceinline__ float exp_f32(float x) { return static_cast<float>(exp(static_cast<double>(x))); }
__device__ __forceinline__ float tanh_f32(float x) { return static_cast<float>(tanh(static_cast<double>(x))); }
__device__ __forceinline__ float cube_f32(float x) {
  double d = static_cast<double>(x);
  return static_cast<float>(d * d * d);
}

// tanh-approximation GELU in the operation order of simulator.py:955-960.
__device__ __forceinline__ float gelu_f32(float x) {
  const float c = 0.7978845608028654f;   // np.float32(np.sqrt(2 / pi))
  const float k = 0.044715f;
  float inner = __fmul_rn(c, __fadd_rn(x, __fmul_rn(k, cube_f32(x))));
  return __fmul_rn(__fmul_rn(x, 0.5f), __fadd_rn(1.0f, tanh_f32(inner)));
}

// ---- NumPy pairwise summation -------------------------------------------------
constexpr int kPwMaxLeaves = 64;

// Leaves of the pairwise tree over n elements, left to right.
__device__ inline int pw_leaves(uint32_t n, uint32_t* loff, uint32_t* llen) {
  uint32_t so[24], sn[24];
  int sp = 0, nl = 0;
  so[sp] = 0;
  sn[sp] = n;
  ++sp;
  while (sp) {
    --sp;
    uint32_t o = so[sp], m = sn[sp];
    if (m <= 128) {
      if (nl < kPwMaxLeaves) { loff[nl] = o; llen[nl] = m; }
      ++nl;
    } else {
      uint32_t h = m / 2;
      h -= h % 8;
      so[sp] = o + h; sn[sp] = m - h; ++sp;   // right (processed second)
      so[sp] = o;     sn[sp] = h;     ++sp;   // left
    }
  }
  return nl;
}

template <class Get>
__device__ inline float pw_leaf(const Get& get, uint32_t o, uint32_t m) {
  if (m < 8) {
    float r = -0.0f;
    for (uint32_t i = 0; i < m; ++i) r = __fadd_rn(r, get(o + i));
    return r;
  }
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = get(o + j);
  uint32_t i = 8;
  for (; i < m - (m % 8); i += 8) {
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], get(o + i + j));
  }
  float res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                        __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
  for (; i < m; ++i) res = __fadd_rn(res, get(o + i));
  return res;
}

// Combines leaf sums in the tree's order (post-order walk of the same split).
__device__ inline float pw_combine(uint32_t n, const float* leaf) {
  uint32_t sn[24];
  uint8_t st[24];
  float vals[24];
  int sp = 0, vp = 0, li = 0;
  sn[sp] = n; st[sp] = 0; ++sp;
  while (sp) {
    uint32_t m = sn[sp - 1];
    if (m <= 128) {
      vals[vp++] = leaf[li++];
      --sp;
      continue;
    }
    uint32_t h = m / 2;
    h -= h % 8;
    if (st[sp - 1] == 0) {
      st[sp - 1] = 1;
      sn[sp] = h; st[sp] = 0; ++sp;
    } else if (st[sp - 1] == 1) {
      st[sp - 1] = 2;
      sn[sp] = m - h; st[sp] = 0; ++sp;
    } else {
      float r = vals[--vp];
      float l = vals[--vp];
      vals[vp++] = __fadd_rn(l, r);
      --sp;
    }
  }
  return vals[0];
}

// Warp-cooperative np.sum(row) for a float32 row of n elements; every lane
// returns the result.  `scratch` holds kPwMaxLeaves*3 words per warp.
// True when the pairwise tree over n elements is perfectly balanced: every
// split halves exactly (n % 16 == 0 above the leaf size), leaving nl <= 8
// leaves of L elements with L a multiple of 8 in [8, 128].
__device__ inline bool pw_balanced(uint32_t n, uint32_t& nl, uint32_t& L) {
  nl = 1;
  L = n;
  while (L > 128) {
    if (L % 16) return false;
    L /= 2;
    nl *= 2;
  }
  return L >= 8 && L % 8 == 0 && nl <= 8;
}

// np.sum of x[0..n) held in shared memory (every lane returns it), or of
// (x[i] - mean)^2 when sq is set.  Balanced trees take the butterfly of
// warp_pairwise_sum without a gather callback; others fall back to it.
template <class Get>
__device__ inline float warp_pairwise_sum(const Get& get, uint32_t n, uint32_t* scratch);

__device__ __forceinline__ float warp_pairwise_sum_smem(const float* x, uint32_t n, uint32_t* scratch,
                                                        bool sq = false, float mean = 0.f,
                                                        uint32_t nz = 0xFFFFFFFFu) {
  // nz (plain sums of non-negative values only): x[nz..n) are +0; adding +0
  // leaves every partial sum as it is, so a leaf stops at nz
  uint32_t bnl, bL;
  if (pw_balanced(n, bnl, bL)) {
    const uint32_t lane = threadIdx.x & 31, leaf = lane >> 2, p = lane & 3;
    float v = 0.f;
    if (leaf < bnl) {
      const float* q = x + leaf * bL + 2 * p;
      float r0, r1;
      if (sq) {
        const float d0 = __fsub_rn(q[0], mean), d1 = __fsub_rn(q[1], mean);
        r0 = __fmul_rn(d0, d0);
        r1 = __fmul_rn(d1, d1);
        for (uint32_t i = 8; i < bL; i += 8) {
          const float e0 = __fsub_rn(q[i], mean), e1 = __fsub_rn(q[i + 1], mean);
          r0 = __fadd_rn(r0, __fmul_rn(e0, e0));
          r1 = __fadd_rn(r1, __fmul_rn(e1, e1));
        }
      } else {
        r0 = q[0];
        r1 = q[1];
        const uint32_t base = leaf * bL + 2 * p;
        for (uint32_t i = 8; i < bL && base + i < nz; i += 8) {
          r0 = __fadd_rn(r0, q[i]);
          r1 = __fadd_rn(r1, q[i + 1]);
        }
      }
      v = __fadd_rn(r0, r1);
    }
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
    for (uint32_t s = 4; s < 4 * bnl; s <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, s));
    return __fadd_rn(0.0f, __shfl_sync(0xffffffffu, v, 0));
  }
  if (sq)
    return warp_pairwise_sum([&](uint32_t j) { const float d = __fsub_rn(x[j], mean); return __fmul_rn(d, d); }, n,
                             scratch);
  return warp_pairwise_sum([&](uint32_t j) { return x[j]; }, n, scratch);
}

// Two rows' np.sum at once (x0[0..n), x1[0..n) in shared memory, non-negative,
// +0 from nz0 / nz1 on): the values of two warp_pairwise_sum_smem calls, the
// two trees' adds interleaved.
__device__ __forceinline__ void warp_pairwise_sum2_smem(const float* x0, const float* x1, uint32_t n,
                                                        uint32_t* scratch0, uint32_t* scratch1, uint32_t nz0,
                                                        uint32_t nz1, float& s0, float& s1) {
  uint32_t bnl, bL;
  if (!pw_balanced(n, bnl, bL)) {
    s0 = warp_pairwise_sum_smem(x0, n, scratch0, false, 0.f, nz0);
    s1 = warp_pairwise_sum_smem(x1, n, scratch1, false, 0.f, nz1);
    return;
  }
  const uint32_t lane = threadIdx.x & 31, leaf = lane >> 2, p = lane & 3;
  float v0 = 0.f, v1 = 0.f;
  if (leaf < bnl) {
    const uint32_t base = leaf * bL + 2 * p;
    const float* q0 = x0 + base;
    const float* q1 = x1 + base;
    float a0 = q0[0], a1 = q0[1], b0 = q1[0], b1 = q1[1];
    const uint32_t nz = nz0 > nz1 ? nz0 : nz1;
    for (uint32_t i = 8; i < bL && base + i < nz; i += 8) {
      if (base + i < nz0) {
        a0 = __fadd_rn(a0, q0[i]);
        a1 = __fadd_rn(a1, q0[i + 1]);
      }
      if (base + i < nz1) {
        b0 = __fadd_rn(b0, q1[i]);
        b1 = __fadd_rn(b1, q1[i + 1]);
      }
    }
    v0 = __fadd_rn(a0, a1);
    v1 = __fadd_rn(b0, b1);
  }
  v0 = __fadd_rn(v0, __shfl_xor_sync(0xffffffffu, v0, 1));
  v1 = __fadd_rn(v1, __shfl_xor_sync(0xffffffffu, v1, 1));
  v0 = __fadd_rn(v0, __shfl_xor_sync(0xffffffffu, v0, 2));
  v1 = __fadd_rn(v1, __shfl_xor_sync(0xffffffffu, v1, 2));
  for (uint32_t sh = 4; sh < 4 * bnl; sh <<= 1) {
    v0 = __fadd_rn(v0, __shfl_xor_sync(0xffffffffu, v0, sh));
    v1 = __fadd_rn(v1, __shfl_xor_sync(0xffffffffu, v1, sh));
  }
  s0 = __fadd_rn(0.0f, __shfl_sync(0xffffffffu, v0, 0));
  s1 = __fadd_rn(0.0f, __shfl_sync(0xffffffffu, v1, 0));
}

template <class Get>
__device__ inline float warp_pairwise_sum(const Get& get, uint32_t n, uint32_t* scratch) {
  const int lane = threadIdx.x & 31;
  uint32_t bnl, bL;
  if (pw_balanced(n, bnl, bL)) {
    // Lanes 4l..4l+3 own leaf l; lane 4l+p runs the leaf's accumulators 2p and
    // 2p+1 in order.  The xor-shuffle butterfly then adds exactly the pairs
    // the tree adds: (r0+r1)+(r2+r3), then the two halves of the leaf, then
    // neighbouring leaves, then neighbouring pairs of leaves.
    const uint32_t leaf = uint32_t(lane) >> 2, p = uint32_t(lane) & 3;
    float v = 0.f;
    if (leaf < bnl) {
      const uint32_t o = leaf * bL + 2 * p;
      float r0 = get(o), r1 = get(o + 1);
      for (uint32_t i = 8; i < bL; i += 8) {
        r0 = __fadd_rn(r0, get(o + i));
        r1 = __fadd_rn(r1, get(o + i + 1));
      }
      v = __fadd_rn(r0, r1);
    }
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 1));
    v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, 2));
    for (uint32_t s = 4; s < 4 * bnl; s <<= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, s));
    return __fadd_rn(0.0f, __shfl_sync(0xffffffffu, v, 0));
  }
  uint32_t* loff = scratch;
  uint32_t* llen = scratch + kPwMaxLeaves;
  float* lsum = reinterpret_cast<float*>(scratch + 2 * kPwMaxLeaves);
  int nl = 0;
  if (lane == 0) nl = pw_leaves(n, loff, llen);
  nl = __shfl_sync(0xffffffffu, nl, 0);
  __syncwarp();
  float total = 0.f;
  if (nl <= kPwMaxLeaves) {
    for (int l = lane; l < nl; l += 32) lsum[l] = pw_leaf(get, loff[l], llen[l]);
    __syncwarp();
    if (lane == 0) total = __fadd_rn(0.0f, pw_combine(n, lsum));
  } else if (lane == 0) {
    // Rows with more leaves than the scratch holds: lane 0 walks the tree.
    uint32_t so[24], sn[24];
    uint8_t st[24];
    float vals[24];
    int sp = 0, vp = 0;
    uint32_t off = 0;
    so[sp] = 0; sn[sp] = n; st[sp] = 0; ++sp;
    while (sp) {
      uint32_t m = sn[sp - 1];
      if (m <= 128) {
        vals[vp++] = pw_leaf(get, so[sp - 1], m);
        --sp;
        continue;
      }
      uint32_t h = m / 2;
      h -= h % 8;
      off = so[sp - 1];
      if (st[sp - 1] == 0) {
        st[sp - 1] = 1;
        so[sp] = off; sn[sp] = h; st[sp] = 0; ++sp;
      } else if (st[sp - 1] == 1) {
        st[sp - 1] = 2;
        so[sp] = off + h; sn[sp] = m - h; st[sp] = 0; ++sp;
      } else {
        float r = vals[--vp];
        float l = vals[--vp];
        vals[vp++] = __fadd_rn(l, r);
        --sp;
      }
    }
    total = __fadd_rn(0.0f, vals[0]);
  }
  total = __shfl_sync(0xffffffffu, total, 0);
  __syncwarp();
  return total;
}

// float32 mean / variance divisor: f32(f64(sum) / n)
__device__ __forceinline__ float div_count(float s, uint32_t n) {
  return static_cast<float>(static_cast<double>(s) / static_cast<double>(n));
}

}  // namespace tac
