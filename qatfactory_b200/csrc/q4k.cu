// Q4_K (GGUF block_q4_K) super-block encoder and decoder for sm_100a.
//
// A super-block is 256 consecutive weights of one row: 8 sub-blocks of 32, each with an
// affine (scale, min) fit whose 6-bit codes ls/lm are quantized against two FP16
// super-block scales d/dmin (qatfactory/quant/formats/q4_k.py:1-17).  The encoder writes
// any of: the reconstruction d*ls*q - dmin*lm in the input dtype, the STE bit mask and the
// 144-byte block [d f16][dmin f16][12 B packed 6-bit scales/mins][128 B nibbles].
//
// Layout: one thread per 32-weight sub-block, 8 consecutive lanes per super-block, so a
// warp covers 4 super-blocks (2 KB of BF16) per pass.  A BF16 sub-block is two 256-bit
// loads and its reconstruction two 256-bit stores; super-block maxima take three
// shuffles.  The level-1 fit is the min-max affine fit (the default "q4_k" format,
// HBM-bound) or the 21-step weighted least-squares search of llama.cpp's
// make_qkx2_quants (FP32-ALU-bound), both kept in registers.
//
// Every float operation repeats the reference's torch CPU expression in the same order:
// `c / t` is t.reciprocal() * c; 32-element sums use torch-CPU's 8-lane vector order
// t[k] = ((v[k] + v[k+8]) + v[k+16]) + v[k+24] then a sequential sum of t[0..7];
// maxima/minima keep the first of equal values (+0 vs -0) and clamp(max=0) keeps -0, as
// torch's CPU reductions and clamp do; the per-weight (x + dm) / deff is an exact
// Markstein quotient.
#include "qatf.h"
#include "qatf_common.cuh"

#include <type_traits>

namespace qatf {

constexpr int kQK = 256;
constexpr int kQ4Threads = 128;
// Minimum resident CTAs per SM the min-max encoder is compiled for (caps its registers):
// writing the reconstruction, and writing blocks only.
#ifndef QATF_Q4K_CTAS
#define QATF_Q4K_CTAS 6
#endif
#ifndef QATF_Q4K_PACK_CTAS
#define QATF_Q4K_PACK_CTAS 8
#endif
constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23: x + kMagic rounds x to an integer, RNE

// (_RMIN + _RDELTA * step + nmax) evaluated in double by Python, then cast to float by
// torch when it multiplies a float tensor (q4_k.py:92-93).
#define QATF_TRIAL(s) ((float)(-1.0 + 0.1 * (double)(s) + 15.0))
__constant__ float c_trial[21] = {QATF_TRIAL(0),  QATF_TRIAL(1),  QATF_TRIAL(2),  QATF_TRIAL(3),  QATF_TRIAL(4),
                                  QATF_TRIAL(5),  QATF_TRIAL(6),  QATF_TRIAL(7),  QATF_TRIAL(8),  QATF_TRIAL(9),
                                  QATF_TRIAL(10), QATF_TRIAL(11), QATF_TRIAL(12), QATF_TRIAL(13), QATF_TRIAL(14),
                                  QATF_TRIAL(15), QATF_TRIAL(16), QATF_TRIAL(17), QATF_TRIAL(18), QATF_TRIAL(19),
                                  QATF_TRIAL(20)};
#undef QATF_TRIAL

// torch.clamp(v, lo, hi): v < lo ? lo : (v > hi ? hi : v); keeps -0.
__device__ __forceinline__ float torch_clamp(float v, float lo, float hi) { return v < lo ? lo : (v > hi ? hi : v); }
// torch.clamp(v, max=0) / torch.minimum(v, 0): a zero keeps its sign.
__device__ __forceinline__ float clamp_max0(float v) { return v > 0.0f ? 0.0f : v; }

// ------------------------------------------------------------------- level 1 fits

// First-wins max / min over the 32 values of a sub-block (torch's CPU reduction).
__device__ __forceinline__ void extrema32(const float* x, float* mx, float* mn) {
  float a = x[0], b = x[0];
#pragma unroll
  for (int i = 1; i < 32; ++i) {
    a = x[i] > a ? x[i] : a;
    b = x[i] < b ? x[i] : b;
  }
  *mx = a;
  *mn = b;
}

// torch-CPU float32 sum of the 32 values f(0..31).
template <typename F>
__device__ __forceinline__ float torch_sum32(F f) {
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < 8; ++k) {
    const float t = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.0f, f(k)), f(k + 8)), f(k + 16)), f(k + 24));
    acc = __fadd_rn(acc, t);
  }
  return acc;
}

// The first-wins minimum given its value: only a zero minimum can differ (+0 vs -0), and
// then it is the first zero of the sub-block.
__device__ __forceinline__ float first_min(const float* x, float value) {
  if (value != 0.0f) return value;
  float z = value;
#pragma unroll
  for (int i = 31; i >= 0; --i) z = x[i] == 0.0f ? x[i] : z;
  return z;
}

// _level1_minmax_torch (q4_k.py:150-163), given the sub-block's max and min values.  The
// max's sign never matters here: a zero max with a positive-zero vmin would need a zero
// first-wins minimum of the other sign, which first-wins rules out.
__device__ __forceinline__ void level1_minmax(const float* x, float xmax, float xmin_value, float* scale,
                                              float* the_min) {
  const float vmin = clamp_max0(first_min(x, xmin_value));
  *scale = __fdiv_rn(__fsub_rn(xmax, vmin), 15.0f);
  *the_min = -vmin;
}

// _level1_grid_search_torch + _make_qkx2 (q4_k.py:139-147, :68-119).
__device__ __forceinline__ void level1_grid(const float* x, float* scale_out, float* min_out) {
  float w[32];
  const float av_x = __fsqrt_rn(__fmul_rn(torch_sum32([&](int i) { return __fmul_rn(x[i], x[i]); }), 0.03125f));
#pragma unroll
  for (int i = 0; i < 32; ++i) w[i] = __fadd_rn(av_x, fabsf(x[i]));
  float xmax, xmin;
  extrema32(x, &xmax, &xmin);
  const float vmin = clamp_max0(xmin);
  const bool degenerate = xmax == vmin;
  const float denom = degenerate ? 1.0f : __fsub_rn(xmax, vmin);
  const float rden = __frcp_rn(denom);          // denom.reciprocal()
  const float iscale = __fmul_rn(rden, 15.0f);  // nmax / denom
  float scale = __frcp_rn(iscale);              // 1.0 / iscale
  float best_error = torch_sum32([&](int i) {
    const float code = torch_clamp(rintf(__fmul_rn(iscale, __fsub_rn(x[i], vmin))), 0.0f, 15.0f);
    const float diff = __fsub_rn(__fadd_rn(__fmul_rn(scale, code), vmin), x[i]);
    return __fmul_rn(__fmul_rn(w[i], diff), diff);
  });
  const float sum_w = torch_sum32([&](int i) { return w[i]; });
  const float sum_x = torch_sum32([&](int i) { return __fmul_rn(w[i], x[i]); });
  float cur_min = vmin;
#pragma unroll 1
  for (int step = 0; step <= 20; ++step) {
    const float trial = __fmul_rn(rden, c_trial[step]);
    float aux[32];
#pragma unroll
    for (int i = 0; i < 32; ++i) aux[i] = torch_clamp(rintf(__fmul_rn(trial, __fsub_rn(x[i], vmin))), 0.0f, 15.0f);
    const float sum_l = torch_sum32([&](int i) { return __fmul_rn(w[i], aux[i]); });
    const float sum_l2 = torch_sum32([&](int i) { return __fmul_rn(__fmul_rn(w[i], aux[i]), aux[i]); });
    const float sum_xl = torch_sum32([&](int i) { return __fmul_rn(__fmul_rn(w[i], aux[i]), x[i]); });
    const float det = __fsub_rn(__fmul_rn(sum_w, sum_l2), __fmul_rn(sum_l, sum_l));
    const float safe_det = det > 0.0f ? det : 1.0f;
    float this_scale = __fdiv_rn(__fsub_rn(__fmul_rn(sum_w, sum_xl), __fmul_rn(sum_x, sum_l)), safe_det);
    float this_min = __fdiv_rn(__fsub_rn(__fmul_rn(sum_l2, sum_x), __fmul_rn(sum_l, sum_xl)), safe_det);
    if (this_min > 0.0f) {
      this_scale = __fdiv_rn(sum_xl, sum_l2 > 0.0f ? sum_l2 : 1.0f);
      this_min = 0.0f;
    }
    const float cur_error = torch_sum32([&](int i) {
      const float d = __fsub_rn(__fadd_rn(__fmul_rn(this_scale, aux[i]), this_min), x[i]);
      return __fmul_rn(__fmul_rn(w[i], d), d);
    });
    if (det > 0.0f && cur_error < best_error) {
      best_error = cur_error;
      scale = this_scale;
      cur_min = this_min;
    }
  }
  *scale_out = degenerate ? 0.0f : scale;
  *min_out = -(degenerate ? vmin : cur_min);
}

// ------------------------------------------------------------------------ level 2

// First-wins max over the 8 sub-blocks of this lane's super-block (lanes 8g..8g+7): the
// value by a shuffle tree, and for a zero maximum the sign of the first zero (torch keeps
// the earlier of +0 / -0).  Called by all 32 lanes.
__device__ __forceinline__ float group_max8(float v, int lane) {
  float m = v;
#pragma unroll
  for (int o = 1; o < 8; o <<= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (!__any_sync(0xffffffffu, m == 0.0f)) return m;
  const uint32_t zeros = (__ballot_sync(0xffffffffu, v == 0.0f) >> (lane & ~7)) & 0xFFu;
  const int first = zeros ? __ffs(zeros) - 1 : 0;
  const float z = __shfl_sync(0xffffffffu, v, (lane & ~7) + first);
  return (m == 0.0f && zeros) ? z : m;
}

struct Level2 {
  float deff, dm;
  uint32_t ls, lm;
  uint16_t d_h, dmin_h;
};

// _level2_encode_torch, scale part (q4_k.py:173-183).  The four super-block divisions
// 1/max_scale, 1/max_min (torch's `63.0 / t` is t.reciprocal() * 63), max_scale/63 and
// max_min/63 are done by lanes 0..3 of the group, one correctly rounded division each, and
// shared by shuffles.  Called by all 32 lanes.
__device__ __forceinline__ Level2 level2(float scale, float the_min, float max_scale, float max_min, int lane) {
  Level2 L;
  const int k = lane & 3;
  const float num = k < 2 ? 1.0f : (k == 2 ? max_scale : max_min);
  const float den = k == 0 ? max_scale : (k == 1 ? max_min : 63.0f);
  const float quo = __fdiv_rn(num, den);
  const int base = lane & ~7;
  const float rcp_scale = __shfl_sync(0xffffffffu, quo, base + 0);
  const float rcp_min = __shfl_sync(0xffffffffu, quo, base + 1);
  const float d_raw = __shfl_sync(0xffffffffu, quo, base + 2);
  const float dmin_raw = __shfl_sync(0xffffffffu, quo, base + 3);
  const float inv_scale = max_scale > 0.0f ? __fmul_rn(rcp_scale, 63.0f) : 0.0f;
  const float inv_min = max_min > 0.0f ? __fmul_rn(rcp_min, 63.0f) : 0.0f;
  const float ls = fminf(fmaxf(rintf(__fmul_rn(inv_scale, scale)), 0.0f), 63.0f);  // integer codes: sign irrelevant
  const float lm = fminf(fmaxf(rintf(__fmul_rn(inv_min, the_min)), 0.0f), 63.0f);
  const __half dh = __float2half_rn(d_raw);
  const __half dmh = __float2half_rn(dmin_raw);
  L.d_h = __half_as_ushort(dh);
  L.dmin_h = __half_as_ushort(dmh);
  L.deff = __fmul_rn(__half2float(dh), ls);
  L.dm = __fmul_rn(__half2float(dmh), lm);
  L.ls = (uint32_t)ls;
  L.lm = (uint32_t)lm;
  return L;
}

// ------------------------------------------------------------------------- encode

// Exact re-encode of one weight (q4_k.py:185-189): reconstruction, code, in-range bit.
__device__ __forceinline__ float encode_exact(const Level2& L, float x, uint32_t* code, uint32_t* in_range) {
  if (L.deff == 0.0f) {
    *code = 0u;
    *in_range = 1u;
    return __fsub_rn(__fmul_rn(L.deff, 0.0f), L.dm);
  }
  const float raw = __fdiv_rn(__fadd_rn(x, L.dm), L.deff);
  const float q = torch_clamp(rintf(raw), 0.0f, 15.0f);
  *code = (uint32_t)q;
  *in_range = (raw >= 0.0f && raw <= 15.0f) ? 1u : 0u;
  return __fsub_rn(__fmul_rn(L.deff, q), L.dm);
}

// Re-encode a whole sub-block.  Fast path (dm > 0, Markstein-exact divisor, every quotient
// >= -15): packed f32x2 arithmetic, rounding by the 1.5*2^23 addition, codes accumulated
// with integer multiply-adds and the mask with funnel shifts.  The quotient is monotonic in
// x, so its extremes come from the sub-block's min and max: when they stay inside
// [-0.5, 15.5) no clamp is needed (RNE already lands in [0, 15]; a -0 code cannot matter with
// dm > 0), and when they stay inside [0, 15] every weight is in range.  Otherwise: the exact
// per-weight path.  x[] is overwritten with the reconstruction; cw[4] receive the nibbles.
__device__ __forceinline__ float markstein(float a, float b, float nb, float y) {
  const float q0 = __fmul_rn(a, y);
  return __fmaf_rn(__fmaf_rn(q0, nb, a), y, q0);
}

template <bool RECON, bool MASK, bool CODES>
__device__ __forceinline__ void encode_subblock(const Level2& L, float xmin, float xmax, float xabs, float* x,
                                                uint32_t* cb, uint32_t* mask) {
  bool fast = L.deff != 0.0f && L.dm > 0.0f;
  BlockDivisor div;
  float qlo = 0.0f, qhi = 0.0f;
  if (fast) {
    div = make_divisor(L.deff, __float_as_uint(__fadd_ru(xabs, L.dm)));
    fast = div.fast;
  }
  if (fast) {
    qlo = markstein(__fadd_rn(xmin, L.dm), L.deff, -L.deff, div.y);
    qhi = markstein(__fadd_rn(xmax, L.dm), L.deff, -L.deff, div.y);
    fast = qlo >= -15.0f;
  }
  if (fast) {
    const float2 dm2 = make_float2(L.dm, L.dm), ndm2 = make_float2(-L.dm, -L.dm);
    const float2 b2 = make_float2(L.deff, L.deff), nb2 = make_float2(-L.deff, -L.deff);
    const float2 y2 = make_float2(div.y, div.y);
    const float2 mg = make_float2(kMagic, kMagic), nmg = make_float2(-kMagic, -kMagic);
    const bool no_clamp = qlo >= -0.5f && qhi < 15.5f;
    const bool all_in = qlo >= 0.0f && qhi <= 15.0f;
    uint32_t m = 0u;
#pragma unroll
    for (int k = 0; k < 8; ++k) cb[k] = 0u;
#pragma unroll
    for (int i = 0; i < 32; i += 2) {
      const float2 a = __fadd2_rn(make_float2(x[i], x[i + 1]), dm2);
      const float2 q0 = __fmul2_rn(a, y2);
      float2 q = __ffma2_rn(__ffma2_rn(q0, nb2, a), y2, q0);
      if (MASK && !all_in) {
        // in range <=> 0 <= q <= 15 <=> bits(q) <= bits(15.0f) (q >= -15, never -0 here)
        m = __funnelshift_l(__float_as_uint(q.x) - 0x41700001u, m, 1);
        m = __funnelshift_l(__float_as_uint(q.y) - 0x41700001u, m, 1);
      }
      if (!no_clamp) q = make_float2(fminf(fmaxf(q.x, 0.0f), 15.0f), fminf(fmaxf(q.y, 0.0f), 15.0f));
      const float2 t = __fadd2_rn(q, mg);   // RNE to an integer
      if (RECON) {
        const float2 r = __fadd2_rn(t, nmg);  // exact
        const float2 rc = __fadd2_rn(__fmul2_rn(b2, r), ndm2);
        x[i] = rc.x;
        x[i + 1] = rc.y;
      }
      if (CODES) {  // bits(t) = bits(1.5 * 2^23) + code: byte i%4 of word i/4, one offset per word
        cb[i >> 2] += __float_as_uint(t.x) * (1u << (8 * (i & 3)));
        cb[i >> 2] += __float_as_uint(t.y) * (1u << (8 * ((i + 1) & 3)));
      }
    }
    if (MASK) *mask = all_in ? 0xFFFFFFFFu : __brev(m);  // element 0 entered first: reverse it to bit 0
    constexpr uint32_t kOff = 0x4B400000u * 0x01010101u;
#pragma unroll
    for (int k = 0; k < 8; ++k) cb[k] -= kOff;
  } else {
    uint32_t m = 0u;
#pragma unroll
    for (int k = 0; k < 8; ++k) cb[k] = 0u;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      uint32_t code, in_range;
      x[i] = encode_exact(L, x[i], &code, &in_range);
      m |= in_range << i;
      cb[i >> 2] |= code << (8 * (i & 3));
    }
    *mask = m;
  }
}

// ------------------------------------------------------------------ loads / stores
// 32 BF16 weights by two 256-bit loads, with their max and min taken on packed halves
// (max/min of BF16 values are exact, and the sign of a zero extremum is settled later by
// first_min); the values are returned as floats.
__device__ __forceinline__ void load32_bf16_extrema(const __nv_bfloat16* p, float* x, float* xmax, float* xmin) {
  uint32_t w[16];
  ld_stream256(p, w);
  ld_stream256(p + 16, w + 8);
  __nv_bfloat162 hi = *reinterpret_cast<const __nv_bfloat162*>(&w[0]), lo = hi;
#pragma unroll
  for (int i = 1; i < 16; ++i) {
    const __nv_bfloat162 v = *reinterpret_cast<const __nv_bfloat162*>(&w[i]);
    hi = __hmax2(hi, v);
    lo = __hmin2(lo, v);
  }
  *xmax = fmaxf(__low2float(hi), __high2float(hi));
  *xmin = fminf(__low2float(lo), __high2float(lo));
#pragma unroll
  for (int i = 0; i < 16; ++i) VecTraits<__nv_bfloat16>::unpack2(w[i], x + 2 * i);
}

template <typename T>
__device__ __forceinline__ void load32(const T* p, bool vec, float* x) {
  using VT = VecTraits<T>;
  if (vec) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      uint32_t w[16];
      ld_stream256(p, w);
      ld_stream256(p + 16, w + 8);
#pragma unroll
      for (int i = 0; i < 16; ++i) VT::unpack2(w[i], x + 2 * i);
    } else {
#pragma unroll
      for (int v = 0; v < 32 / VT::kVec; ++v) VT::to_float(ld_stream(p + v * VT::kVec), x + v * VT::kVec);
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) x[i] = VT::load1(p + i);
  }
}

template <typename T>
__device__ __forceinline__ void store32(T* p, bool vec, const float* x) {
  using VT = VecTraits<T>;
  if (vec) {
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      uint32_t w[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = pack_bf16x2(x[2 * i], x[2 * i + 1]);
      st256(p, w);
      st256(p + 16, w + 8);
    } else {
#pragma unroll
      for (int v = 0; v < 32 / VT::kVec; ++v) st_v4(p + v * VT::kVec, VT::from_float(x + v * VT::kVec));
    }
  } else {
#pragma unroll
    for (int i = 0; i < 32; ++i) VT::store1(p + i, x[i]);
  }
}

// ------------------------------------------------------------------------- encoder
// OUT selects the outputs at compile time (kQ4Recon | kQ4Mask | kQ4Blocks); kQ4Runtime
// writes whichever of recon / mask / blocks is non-null.
constexpr int kQ4Recon = 1, kQ4Mask = 2, kQ4Blocks = 4, kQ4Runtime = 8;

template <typename T, int METHOD, int OUT>
__global__ void __launch_bounds__(kQ4Threads, METHOD == QATF_Q4K_MINMAX ? (OUT == kQ4Blocks ? QATF_Q4K_PACK_CTAS : QATF_Q4K_CTAS) : 1)
    q4k_encode_kernel(const T* __restrict__ x, int64_t n_sb,
                                                                int64_t sb_per_row, int64_t ld, bool vec_in,
                                                                bool vec_out, T* __restrict__ recon,
                                                                uint8_t* __restrict__ mask,
                                                                uint8_t* __restrict__ blocks) {
  constexpr bool kRT = (OUT & kQ4Runtime) != 0;
  const bool want_recon = kRT ? recon != nullptr : (OUT & kQ4Recon) != 0;
  const bool want_mask = kRT ? mask != nullptr : (OUT & kQ4Mask) != 0;
  const bool want_blocks = kRT ? blocks != nullptr : (OUT & kQ4Blocks) != 0;
  pdl_wait();  // launched with programmatic dependent launch: nothing is read before this
  pdl_launch_dependents();
  const int lane = threadIdx.x & 31;
  const int j = lane & 7;  // sub-block within the super-block
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t sb0 = warp * 4; sb0 < n_sb; sb0 += n_warps * 4) {
    const int64_t sb = sb0 + (lane >> 3);
    const bool live = sb < n_sb;
    float xs[32];
    float scale, the_min, xmin = 0.0f, xmax = 0.0f;
    if (live) {
      const T* src = x + sb * kQK + j * 32;
      if (ld != sb_per_row * kQK) {  // strided rows
        const int64_t row = sb / sb_per_row, kb = sb - row * sb_per_row;
        src = x + row * ld + kb * kQK + j * 32;
      }
      if (std::is_same<T, __nv_bfloat16>::value && vec_in) {
        load32_bf16_extrema(reinterpret_cast<const __nv_bfloat16*>(src), xs, &xmax, &xmin);
      } else {
        load32(src, vec_in, xs);
        xmin = xmax = xs[0];
#pragma unroll
        for (int i = 1; i < 32; ++i) {
          xmin = fminf(xmin, xs[i]);
          xmax = fmaxf(xmax, xs[i]);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 32; ++i) xs[i] = 0.0f;
    }
    const float xabs = fmaxf(fabsf(xmin), fabsf(xmax));
    if constexpr (METHOD == QATF_Q4K_MINMAX) {
      level1_minmax(xs, xmax, xmin, &scale, &the_min);
    } else {
      level1_grid(xs, &scale, &the_min);
    }
    const float max_scale = group_max8(scale, lane);
    const float max_min = group_max8(the_min, lane);
    const Level2 L = level2(scale, the_min, max_scale, max_min, lane);
    uint32_t cb[8], bits = 0u;
    if (kRT) {
      encode_subblock<true, true, true>(L, xmin, xmax, xabs, xs, cb, &bits);
    } else {
      encode_subblock<(OUT & kQ4Recon) != 0, (OUT & kQ4Mask) != 0, (OUT & kQ4Blocks) != 0>(L, xmin, xmax, xabs, xs,
                                                                                           cb, &bits);
    }
    const int64_t e0 = sb * kQK + j * 32;
    if (live && want_recon) store32(recon + e0, vec_out, xs);
    if (live && want_mask) reinterpret_cast<uint32_t*>(mask)[e0 >> 5] = bits;
    if (want_blocks) {
      // block_q4_K = [d f16][dmin f16][12 scale bytes][128 B qs], 16-byte aligned.  qs[g*32 + i]
      // = code(2g, i) | code(2g+1, i) << 4 (q4_k.py:304-315): the even lane of each sub-block
      // pair stores those 32 bytes.  Scale byte 4+j, 8+j and 12+j (q4_k.py:286-301) come from
      // lane j < 4, combining its own ls/lm with those of lane j+4; lane 0 gathers them and
      // stores the 16-byte header.
      uint32_t ob[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) ob[k] = __shfl_down_sync(0xffffffffu, cb[k], 1);
      const uint32_t ls_hi = __shfl_down_sync(0xffffffffu, L.ls, 4);
      const uint32_t lm_hi = __shfl_down_sync(0xffffffffu, L.lm, 4);
      const uint32_t trio = ((L.ls & 0x3Fu) | ((ls_hi >> 4) << 6)) | (((L.lm & 0x3Fu) | ((lm_hi >> 4) << 6)) << 8) |
                            (((ls_hi & 0xFu) | ((lm_hi & 0xFu) << 4)) << 16);
      const uint32_t t1 = __shfl_down_sync(0xffffffffu, trio, 1);
      const uint32_t t2 = __shfl_down_sync(0xffffffffu, trio, 2);
      const uint32_t t3 = __shfl_down_sync(0xffffffffu, trio, 3);
      if (live) {
        uint8_t* blk = blocks + sb * 144;
        if ((j & 1) == 0) {
          uint4* dst = reinterpret_cast<uint4*>(blk + 16 + (j >> 1) * 32);
          dst[0] = make_uint4(cb[0] | (ob[0] << 4), cb[1] | (ob[1] << 4), cb[2] | (ob[2] << 4), cb[3] | (ob[3] << 4));
          dst[1] = make_uint4(cb[4] | (ob[4] << 4), cb[5] | (ob[5] << 4), cb[6] | (ob[6] << 4), cb[7] | (ob[7] << 4));
        }
        if (j == 0) {
          const uint32_t lo01 = __byte_perm(trio, t1, 0x5140u);  // bytes: trio.0, t1.0, trio.1, t1.1
          const uint32_t lo23 = __byte_perm(t2, t3, 0x5140u);
          const uint32_t hi01 = __byte_perm(trio, t1, 0x0062u);  // trio.2, t1.2
          const uint32_t hi23 = __byte_perm(t2, t3, 0x0062u);
          *reinterpret_cast<uint4*>(blk) =
              make_uint4((uint32_t)L.d_h | ((uint32_t)L.dmin_h << 16), __byte_perm(lo01, lo23, 0x5410u),
                         __byte_perm(lo01, lo23, 0x7632u), __byte_perm(hi01, hi23, 0x5410u));
        }
      }
    }
  }
}

// ------------------------------------------------------------------------ dequant
// dequantize_q4_k (q4_k.py:359-385): one warp per super-block, 8 outputs per lane.
__global__ void __launch_bounds__(256) q4k_dequant_kernel(const uint8_t* __restrict__ blocks, int64_t n_sb,
                                                          float* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int64_t warp = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int64_t n_warps = ((int64_t)gridDim.x * blockDim.x) >> 5;
  for (int64_t sb = warp; sb < n_sb; sb += n_warps) {
    const uint8_t* b = blocks + sb * 144;
    const float d = __half2float(__ushort_as_half((uint16_t)(b[0] | (b[1] << 8))));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(b[2] | (b[3] << 8))));
    const int j = lane >> 2;  // sub-block of this lane's 8 weights
    const uint8_t* s = b + 4;
    uint32_t ls, lm;
    if (j < 4) {
      ls = s[j] & 0x3Fu;
      lm = s[j + 4] & 0x3Fu;
    } else {
      ls = (s[j + 4] & 0xFu) | (((uint32_t)(s[j - 4] >> 6) & 3u) << 4);
      lm = (uint32_t)(s[j + 4] >> 4) | (((uint32_t)(s[j] >> 6) & 3u) << 4);
    }
    const float deff = __fmul_rn(d, (float)ls), dm = __fmul_rn(dmin, (float)lm);
    const int e0 = lane * 8;
    const int g = e0 / 64, o = e0 % 64;
    const uint8_t* q = b + 16 + g * 32 + (o % 32);
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t code = o < 32 ? (q[i] & 0xFu) : (q[i] >> 4);
      v[i] = __fsub_rn(__fmul_rn(deff, (float)code), dm);
    }
    float4* dst = reinterpret_cast<float4*>(out + sb * kQK + e0);
    dst[0] = make_float4(v[0], v[1], v[2], v[3]);
    dst[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// The same with coalesced stores: thread f writes the float4 of super-block f / 64, elements
// e = 4 (f % 64) .. +3 of sub-block j = e / 32, reading the block's 16-byte header (shared by
// the 64 threads of the block through L1) and the four code bytes qs[(j/2)*32 + e%32 ..]
// (low nibbles for even j, high for odd).
__global__ void __launch_bounds__(256) q4k_dequant_vec_kernel(const uint8_t* __restrict__ blocks, int64_t n_sb,
                                                              float4* __restrict__ out) {
  const int64_t n4 = n_sb * 64;
  for (int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; f < n4; f += (int64_t)gridDim.x * blockDim.x) {
    const int64_t sb = f >> 6;
    const int e = (int)(f & 63) * 4;
    const int j = e >> 5;
    const uint8_t* b = blocks + sb * 144;
    const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(b));
    const uint32_t qw = __ldg(reinterpret_cast<const uint32_t*>(b + 16 + (j >> 1) * 32 + (e & 31)));
    const float d = __half2float(__ushort_as_half((uint16_t)(hdr.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(hdr.x >> 16)));
    // scale bytes s[0..11] are header bytes 4..15 = words hdr.y, hdr.z, hdr.w (q4_k.py:343-356)
    const uint32_t sw[3] = {hdr.y, hdr.z, hdr.w};
    auto sbyte = [&](int k) { return (sw[k >> 2] >> (8 * (k & 3))) & 0xFFu; };
    uint32_t ls, lm;
    if (j < 4) {
      ls = sbyte(j) & 0x3Fu;
      lm = sbyte(j + 4) & 0x3Fu;
    } else {
      ls = (sbyte(j + 4) & 0xFu) | ((sbyte(j - 4) >> 6) << 4);
      lm = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
    }
    const float deff = __fmul_rn(d, (float)ls), dm = __fmul_rn(dmin, (float)lm);
    const int sh = (j & 1) * 4;
    float v[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __fsub_rn(__fmul_rn(deff, (float)((qw >> (8 * i + sh)) & 0xFu)), dm);
    out[f] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

// The same with 32-byte stores: thread f writes the 8 floats e = 8 (f % 32) .. +7 of
// super-block f / 32 (one st.global.v8), from an 8-byte load of their codes (gate weight of
// configuration 3: 49.5 -> 43.2 us against the 16-byte-store kernel above, which serves outputs
// that are only 16-byte aligned).
__global__ void __launch_bounds__(256) q4k_dequant_v8_kernel(const uint8_t* __restrict__ blocks, int64_t n_sb,
                                                             float* __restrict__ out) {
  const int64_t n8 = n_sb * 32;
  for (int64_t f = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; f < n8; f += (int64_t)gridDim.x * blockDim.x) {
    const int64_t sb = f >> 5;
    const int e = (int)(f & 31) * 8;
    const int j = e >> 5;
    const uint8_t* b = blocks + sb * 144;
    const uint4 hdr = __ldg(reinterpret_cast<const uint4*>(b));
    const uint2 qw = __ldg(reinterpret_cast<const uint2*>(b + 16 + (j >> 1) * 32 + (e & 31)));
    const float d = __half2float(__ushort_as_half((uint16_t)(hdr.x & 0xFFFFu)));
    const float dmin = __half2float(__ushort_as_half((uint16_t)(hdr.x >> 16)));
    const uint32_t sw[3] = {hdr.y, hdr.z, hdr.w};
    auto sbyte = [&](int k) { return (sw[k >> 2] >> (8 * (k & 3))) & 0xFFu; };
    uint32_t ls, lm;
    if (j < 4) {
      ls = sbyte(j) & 0x3Fu;
      lm = sbyte(j + 4) & 0x3Fu;
    } else {
      ls = (sbyte(j + 4) & 0xFu) | ((sbyte(j - 4) >> 6) << 4);
      lm = (sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4);
    }
    const float deff = __fmul_rn(d, (float)ls), dm = __fmul_rn(dmin, (float)lm);
    const int sh = (j & 1) * 4;
    uint32_t v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t word = i < 4 ? qw.x : qw.y;
      v[i] = __float_as_uint(__fsub_rn(__fmul_rn(deff, (float)((word >> (8 * (i & 3) + sh)) & 0xFu)), dm));
    }
    st256(out + f * 8, v);
  }
}

template <typename F>
int q4_dispatch(int dtype, F&& f) {
  switch (dtype) {
    case kF32:
      return f(float{});
    case kF16:
      return f(__half{});
    case kBF16:
      return f(__nv_bfloat16{});
    default:
      return QATF_ERR_DTYPE;
  }
}

}  // namespace qatf

using namespace qatf;

extern "C" int qatf_q4k_encode(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, int method, void* recon,
                               uint8_t* mask_bits, uint8_t* blocks, void* stream) {
  if (rows < 0 || cols < 0 || cols % kQK != 0 || ld < cols) return QATF_ERR_INVALID;
  if (method != QATF_Q4K_GRID_SEARCH && method != QATF_Q4K_MINMAX) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (x == nullptr) return QATF_ERR_INVALID;
  if (blocks != nullptr && (reinterpret_cast<uintptr_t>(blocks) & 15u) != 0) return QATF_ERR_INVALID;
  if (mask_bits != nullptr && (reinterpret_cast<uintptr_t>(mask_bits) & 3u) != 0) return QATF_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t sb_per_row = cols / kQK;
  const int64_t n_sb = rows * sb_per_row;
  return q4_dispatch(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    const int64_t align = std::is_same<T, __nv_bfloat16>::value ? 32 : 16;
    const bool vec_in = (reinterpret_cast<uintptr_t>(x) % align == 0) && ((ld * (int64_t)sizeof(T)) % align == 0);
    const bool vec_out = recon != nullptr && (reinterpret_cast<uintptr_t>(recon) % align == 0);
    const T* xt = static_cast<const T*>(x);
    T* rt = static_cast<T*>(recon);
    auto run = [&](auto kernel) {
      // consecutive tensors (one layer's linears after another) overlap launch and tail
      launch_pdl(kernel, dim3((unsigned)persistent_grid(n_sb * 8, (const void*)kernel, kQ4Threads)), dim3(kQ4Threads),
                 s, xt, n_sb, sb_per_row, ld, vec_in, vec_out, rt, mask_bits, blocks);
      return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
    };
    if (method == QATF_Q4K_GRID_SEARCH) return run(q4k_encode_kernel<T, QATF_Q4K_GRID_SEARCH, kQ4Runtime>);
    // min-max: the three output sets the quant API asks for are specialised
    const int out = (recon != nullptr ? kQ4Recon : 0) | (mask_bits != nullptr ? kQ4Mask : 0) |
                    (blocks != nullptr ? kQ4Blocks : 0);
    switch (out) {
      case kQ4Recon | kQ4Mask:
        return run(q4k_encode_kernel<T, QATF_Q4K_MINMAX, kQ4Recon | kQ4Mask>);
      case kQ4Blocks:
        return run(q4k_encode_kernel<T, QATF_Q4K_MINMAX, kQ4Blocks>);
      case kQ4Recon | kQ4Blocks:
        return run(q4k_encode_kernel<T, QATF_Q4K_MINMAX, kQ4Recon | kQ4Blocks>);
      default:
        return run(q4k_encode_kernel<T, QATF_Q4K_MINMAX, kQ4Runtime>);
    }
  });
}

extern "C" int qatf_q4k_dequant(const uint8_t* blocks, int64_t rows, int64_t cols, float* out, void* stream) {
  if (rows < 0 || cols < 0 || cols % kQK != 0) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (blocks == nullptr || out == nullptr || !aligned16(out)) return QATF_ERR_INVALID;
  const int64_t n_sb = rows * (cols / kQK);
  if (aligned16(blocks) && aligned32(out)) {
    auto kv = q4k_dequant_v8_kernel;
    q4k_dequant_v8_kernel<<<persistent_grid(n_sb * 32, (const void*)kv, 256), 256, 0,
                            static_cast<cudaStream_t>(stream)>>>(blocks, n_sb, out);
    return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
  }
  if (aligned16(blocks)) {
    auto kv = q4k_dequant_vec_kernel;
    q4k_dequant_vec_kernel<<<persistent_grid(n_sb * 64, (const void*)kv, 256), 256, 0,
                             static_cast<cudaStream_t>(stream)>>>(blocks, n_sb, reinterpret_cast<float4*>(out));
    return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
  }
  auto k = q4k_dequant_kernel;
  q4k_dequant_kernel<<<persistent_grid(n_sb * 32, (const void*)k, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      blocks, n_sb, out);
  return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
}
