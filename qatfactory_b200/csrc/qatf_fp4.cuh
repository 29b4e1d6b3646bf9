// NVFP4 / MXFP4 block arithmetic shared by the quantization kernels (fp4.cu) and the W4A4
// GEMM whose producer side quantizes its activation operand (gemm.cu): block scales, exact
// quotients, the hardware E2M1 / E4M3 converters, and the BF16 block-per-thread fast path.
// Every function here reproduces the reference torch arithmetic bit for bit
// (qatfactory/quant/formats/nvfp4.py:44-121, :400-501; mxfp4.py:48-174).
#pragma once

#include "qatf.h"
#include "qatf_common.cuh"

namespace qatf {

enum Fp4Mode : int { kNV = 0, kMXEven = 1, kMXCeil = 2 };

template <int MODE>
struct Fp4Consts {
  static constexpr int kBlock = MODE == kNV ? 16 : 32;
};

// Launch-wide NVFP4 state: the global scale tensor_amax / 2688 (nvfp4.py:483) and the
// reference's zero-amax branch (nvfp4.py:493-494).
struct NvGlobal {
  float gs;
  bool zero;
  float denom;   // gs * 6
  float rdenom;  // RN(1 / denom), for Markstein quotients block_amax / denom
  bool denom_ok; // denom in [2^-100, 2^100]
};

__device__ __forceinline__ NvGlobal nv_global(const float* tensor_amax) {
  NvGlobal g;
  float a = __ldg(tensor_amax);
  g.zero = (a == 0.0f);
  g.gs = __fdiv_rn(a, 2688.0f);
  g.denom = __fmul_rn(g.gs, 6.0f);
  g.rdenom = __frcp_rn(g.denom);
  const uint32_t e = (__float_as_uint(g.denom) >> 23) & 0xFFu;
  g.denom_ok = (__float_as_uint(g.denom) >> 31) == 0u && e >= 27u && e <= 227u;
  return g;
}

// Per-block scale state.
struct Fp4Block {
  float scale;  // dequant scale: NVFP4 block_scale * global_scale, MXFP4 2^k
  float inv;    // MXFP4: 2^-k (x * 2^-k == x / 2^k exactly)
  float lim;    // in_range <=> |x| <= lim
  BlockDivisor div;
  uint32_t byte;  // stored scale byte (E4M3 for NVFP4, biased E8M0 for MXFP4)
  bool zero;      // output forced to +0 (NVFP4 zero tensor amax, MXFP4 CEIL zero block)
};

template <int MODE>
__device__ __forceinline__ Fp4Block fp4_block(uint32_t amax_bits, const NvGlobal& g) {
  Fp4Block p;
  if constexpr (MODE == kNV) {
    // nvfp4.py:483-491: bs = e4m3(block_amax / (gs * 6)), 0 -> 2^-9, ds = bs * gs
    float q = __fdiv_rn(__uint_as_float(amax_bits), __fmul_rn(g.gs, 6.0f));
    uint32_t byte;
    float bs = e4m3_rne(q, &byte);
    if (bs == 0.0f) {
      bs = 0.001953125f;
      byte = 1u;
    }
    p.scale = __fmul_rn(bs, g.gs);
    p.lim = __fmul_rn(p.scale, 6.0f);
    p.div = make_divisor(p.scale, amax_bits);
    p.inv = 0.0f;
    p.byte = byte;
    p.zero = g.zero;
  } else if constexpr (MODE == kMXEven) {
    int k = e8m0_exponent_even(amax_bits);  // mxfp4.py:48-60
    p.scale = pow2i(k);
    p.inv = pow2i(-k);
    p.lim = __fmul_rn(p.scale, 6.0f);
    p.byte = (uint32_t)(k + 127);
    p.zero = false;
  } else {
    int biased = e8m0_biased_ceil(__uint_as_float(amax_bits));  // mxfp4.py:73-98
    p.scale = pow2i(biased - 127);
    p.inv = pow2i(127 - biased);
    p.lim = __int_as_float(0x7F800000);
    p.byte = (uint32_t)biased;
    p.zero = biased == 0;
  }
  return p;
}


// float -> float8_e4m3fn -> float of a value in [0, inf), by the hardware converter
// (round to nearest even, subnormals in units of 2^-9, saturating at 448 like the
// reference's clamp before the cast).  Returns the value and the stored byte.
__device__ __forceinline__ float e4m3_hw(float v, uint32_t* byte_out) {
  uint16_t b;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(b) : "f"(v), "f"(0.0f));
  uint32_t h;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(b));
  *byte_out = b & 0xFFu;
  return __half2float(__ushort_as_half((uint16_t)(h & 0xFFFFu)));
}

// Fp4Block of an NVFP4 block for the bf16 path: identical values to fp4_block<kNV>, with
// block_amax / (gs * 6) as a Markstein quotient and the E4M3 cast in hardware when both are
// provably exact (finite amax, no under/overflow); otherwise the scalar path.
__device__ __forceinline__ Fp4Block nv_block_hw(uint32_t amax_bits, const NvGlobal& g) {
  const float bamax = __uint_as_float(amax_bits);
  const int gap = (int)(amax_bits >> 23) - (int)((__float_as_uint(g.denom) >> 23) & 0xFFu);
  const bool ok = g.denom_ok && amax_bits < 0x7F800000u && (amax_bits == 0u || amax_bits >= 0x0D800000u) && gap <= 125;
  if (!ok) return fp4_block<kNV>(amax_bits, g);
  Fp4Block p;
  const float q0 = __fmul_rn(bamax, g.rdenom);
  const float q = __fmaf_rn(__fmaf_rn(-q0, g.denom, bamax), g.rdenom, q0);
  uint32_t byte;
  float bs = e4m3_hw(q, &byte);
  if (bs == 0.0f) {
    bs = 0.001953125f;
    byte = 1u;
  }
  p.scale = __fmul_rn(bs, g.gs);
  p.lim = __fmul_rn(p.scale, 6.0f);
  p.div = make_divisor(p.scale, amax_bits);
  p.inv = 0.0f;
  p.byte = byte;
  p.zero = g.zero;
  return p;
}

template <int MODE>
__device__ __forceinline__ Fp4Block fp4_block_bf16(uint32_t amax_bits, const NvGlobal& g) {
  if constexpr (MODE == kNV) {
    return nv_block_hw(amax_bits, g);
  } else {
    return fp4_block<MODE>(amax_bits, g);
  }
}

// Signed E2M1 code value of one element: _round_to_e2m1(clamp(x / scale, -6, 6)).
template <int MODE>
__device__ __forceinline__ float fp4_code(const Fp4Block& p, float v) {
  float n = (MODE == kNV) ? divide(p.div, v) : __fmul_rn(v, p.inv);
  return e2m1_round(n);
}

// Canonical nibble of a signed code value (nvfp4.py:67-73): sign << 3 | level, -0 -> 0.
__device__ __forceinline__ uint32_t fp4_nibble(float code) {
  uint32_t idx = e2m1_index(fabsf(code));
  uint32_t neg = (code < 0.0f && idx != 0u) ? 8u : 0u;
  return neg | idx;
}

template <int MODE>
__device__ __forceinline__ NvGlobal load_global(const float* tensor_amax) {
  if constexpr (MODE == kNV) {
    return nv_global(tensor_amax);
  } else {
    NvGlobal g;
    g.gs = 0.0f;
    g.zero = false;
    g.denom = g.rdenom = 0.0f;
    g.denom_ok = false;
    return g;
  }
}


// ------------------------------------------------------------ bf16 fast path
// For BF16 inputs the per-element work is done on packed 16-bit halves and by the
// hardware E2M1 converter, which rounds to nearest even and saturates at +-6 exactly
// like the reference's clamp + bucketize.  The converter is fed the signed quotient
// x / scale, so the code's sign comes out of the converter: a nonzero negative element
// whose code rounds to zero gives -0, as torch's sign() * level does, and a zero of
// either sign gives +0 because the quotient of +-0 is formed as a sum with +0 (the last
// FMA of the Markstein sequence for NVFP4, x * 2^-k + 0 when packing MXFP4), matching
// torch.sign(+-0) == 0.  MXFP4 fake quantization instead feeds magnitudes and ORs in the
// input's sign bit for nonzero inputs (measured 1-2% faster in that latency-bound kernel).
// A block takes this path only where it is provably exact:
//   MXFP4: finite amax and 2^k in [2^-120, 2^16], so x * 2^-k is exact and nonzero for
//          every nonzero x and the reconstruction code * 2^k is exact;
//   NVFP4: finite amax, a Markstein-exact divisor ds in [2^-96, 2^26].  Elements with
//          |x| >= 2^-100 get RN(x / ds) exactly; an element with 0 < |x| < 2^-100 gets a
//          quotient of the right sign whose magnitude stays below 2^-3 (both Markstein
//          terms are below 2^-4), so it rounds to the same signed zero code as the exact
//          quotient would.
// Other blocks fall back to the per-element path above.

// E2M1 codes of two floats as an f16x2 of the signed code values (lo in the low half).
__device__ __forceinline__ uint32_t e2m1x2_to_f16x2(float lo, float hi) {
  uint32_t h;
  asm("{\n\t.reg .b8 t;\n\tcvt.rn.satfinite.e2m1x2.f32 t, %2, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}"
      : "=r"(h)
      : "f"(lo), "f"(hi));
  return h;
}

// E2M1 codes of eight floats: the packed word (element 2i in the low nibble of byte i, signs
// as the converter gives them) and the four f16x2 code pairs.
__device__ __forceinline__ uint32_t e2m1x8(const float2* n, uint32_t* h) {
  uint32_t word;
  asm("{\n\t.reg .b8 t0, t1, t2, t3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t0, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t1, %8, %7;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t2, %10, %9;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t3, %12, %11;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, t0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, t1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, t2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %4, t3;\n\t"
      "mov.b32 %0, {t0, t1, t2, t3};\n\t}"
      : "=r"(word), "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
      : "f"(n[0].x), "f"(n[0].y), "f"(n[1].x), "f"(n[1].y), "f"(n[2].x), "f"(n[2].y), "f"(n[3].x), "f"(n[3].y));
  return word;
}

// The packed word alone.
__device__ __forceinline__ uint32_t e2m1x8_word(const float2* n) {
  uint32_t word;
  asm("{\n\t.reg .b8 t0, t1, t2, t3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 t3, %8, %7;\n\t"
      "mov.b32 %0, {t0, t1, t2, t3};\n\t}"
      : "=r"(word)
      : "f"(n[0].x), "f"(n[0].y), "f"(n[1].x), "f"(n[1].y), "f"(n[2].x), "f"(n[2].y), "f"(n[3].x), "f"(n[3].y));
  return word;
}

// Stored nibbles of a word of eight signed E2M1 codes: a code of magnitude 0 is stored as +0
// (nvfp4.py:72), so bit 3 of a nibble survives only where its magnitude bits are nonzero
// (magnitude + 7 carries into bit 3 exactly then, and never into the next nibble).
__device__ __forceinline__ uint32_t e2m1_canonical(uint32_t word) {
  return word & (((word & 0x77777777u) + 0x77777777u) | 0x77777777u);
}

__device__ __forceinline__ uint32_t max_u16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.u16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Bit mask of in-range elements of 4 words (8 elements): bit 15 of each half of
// d[i] = (lim16 | 0x8000) * 0x10001 - |x| is set iff that |x| <= lim (a 16-bit compare with
// no borrow between halves).  prmt gathers the high byte of every half (element order),
// and one multiply moves the four byte MSBs of a word into bits 28..31.
__device__ __forceinline__ uint32_t gather_half_msbs(const uint32_t* d) {
  const uint32_t a = __byte_perm(d[0], d[1], 0x7531u) & 0x80808080u;
  const uint32_t c = __byte_perm(d[2], d[3], 0x7531u) & 0x80808080u;
  return ((a * 0x00204081u) >> 28) | (((c * 0x00204081u) >> 24) & 0xF0u);
}

// Per-block parameters of the bf16 fast path, from the block amax as bf16 bits.
struct Bf16Block {
  float scale, inv;  // MX: 2^k and 2^-k; NVFP4: ds and RN(1/ds)
  float nscale;      // -scale (the Markstein residual's multiplier)
  uint32_t limx;     // replicated 16-bit in-range limit (see gather_half_msbs)
  bool fast;
};

template <int MODE>
__device__ __forceinline__ Bf16Block bf16_block(uint32_t amax16, const Fp4Block& p) {
  Bf16Block b;
  b.scale = p.scale;
  b.nscale = -p.scale;
  if constexpr (MODE == kNV) {
    b.inv = p.div.y;
    b.fast = p.div.fast && __float_as_uint(p.scale) >= 0x0F800000u && amax16 < 0x7F80u && !p.zero;
  } else {
    b.inv = p.inv;
    const int e = (int)((__float_as_uint(p.scale) >> 23) & 0xFFu);  // 2^k normal: e = k + 127
    b.fast = amax16 < 0x7F80u && e >= 7 && e <= 143 && !p.zero;
  }
  const uint32_t lim16 = __float_as_uint(p.lim) >> 16;  // |x| <= lim  <=>  bf16(|x|) bits <= lim16
  b.limx = (lim16 | 0x8000u) * 0x00010001u;
  return b;
}

// ------------------------------------------------------------ NVFP4 scale table
// What an NVFP4 block's fast path needs beyond its E4M3 scale byte depends only on that byte
// and the tensor's global scale gs: ds = bs * gs, RN(1 / ds), the in-range bound 6 ds as a
// replicated 16-bit BF16 limit, and whether ds lies where the Markstein quotient is exact.  A
// CTA builds these for all 128 non-negative bytes once (128 correctly rounded reciprocals),
// and a block then costs one shared-memory load after its E4M3 conversion instead of the
// decode, the reciprocal and the range checks.  Values are those of nv_block_hw +
// make_divisor + bf16_block<kNV>, bit for bit.
struct NvScaleEntry {
  float scale, inv;  // ds and RN(1 / ds)
  uint32_t limx;     // see Bf16Block::limx
  uint32_t meta;     // bit 31: ds in [2^-96, 2^26]; bits 0..7: the biased exponent of ds
};
constexpr int kNvTableEntries = 128;

// Fills t[0..127] (byte 0 stands for byte 1: a zero scale is stored as 2^-9, nvfp4.py:487-489).
// Every thread of the CTA calls it; it ends with a CTA barrier.
__device__ __forceinline__ void nv_table_build(NvScaleEntry* t, const NvGlobal& g) {
  for (int i = threadIdx.x; i < kNvTableEntries; i += blockDim.x) {
    const uint16_t byte = (uint16_t)(i == 0 ? 1 : i);
    uint32_t h;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h) : "h"(byte));
    const float bs = __half2float(__ushort_as_half((uint16_t)(h & 0xFFFFu)));
    NvScaleEntry e;
    e.scale = __fmul_rn(bs, g.gs);
    e.inv = __frcp_rn(e.scale);
    const uint32_t sb = __float_as_uint(e.scale);
    e.limx = (((__float_as_uint(__fmul_rn(e.scale, 6.0f)) >> 16) | 0x8000u)) * 0x00010001u;
    e.meta = ((sb >= 0x0F800000u && sb <= 0x4C800000u) ? 0x80000000u : 0u) | (sb >> 23);
    t[i] = e;
  }
  __syncthreads();
}

// The fast-path parameters of an NVFP4 block from the table, and its stored scale byte.
// Returns false where the block needs the scalar path (b and byte are then unset): a zero or
// extreme tensor amax, a non-finite or tiny block amax, or a divisor outside the exact range,
// exactly the blocks for which nv_block_hw / bf16_block<kNV> do not give b.fast.
__device__ __forceinline__ bool nv_block_table(uint32_t m16, const NvGlobal& g, const NvScaleEntry* t, Bf16Block& b,
                                               uint32_t& byte) {
  const uint32_t amax_bits = m16 << 16;
  const int aexp = (int)(amax_bits >> 23);
  const int gap = aexp - (int)((__float_as_uint(g.denom) >> 23) & 0xFFu);
  if (!(g.denom_ok && !g.zero && m16 < 0x7F80u && (amax_bits == 0u || amax_bits >= 0x0D800000u) && gap <= 125))
    return false;
  const float bamax = __uint_as_float(amax_bits);
  const float q0 = __fmul_rn(bamax, g.rdenom);
  const float q = __fmaf_rn(__fmaf_rn(-q0, g.denom, bamax), g.rdenom, q0);
  uint16_t cv;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %2, %1;" : "=h"(cv) : "f"(q), "f"(0.0f));
  const uint32_t raw = cv & 0x7Fu;  // q >= 0: the sign bit is clear and satfinite stops at 0x7E
  const NvScaleEntry e = t[raw];
  byte = raw == 0u ? 1u : raw;
  b.scale = e.scale;
  b.nscale = -e.scale;
  b.inv = e.inv;
  b.limx = e.limx;
  b.fast = (e.meta >> 31) != 0u && aexp - (int)(e.meta & 0xFFu) <= 125;
  return b.fast;
}

// Signed x / scale of a pair of elements, with +-0 -> +0: a Markstein quotient with packed
// f32x2 arithmetic (NVFP4) or an exact multiply by 2^-k plus +0 (MXFP4).
template <int MODE>
__device__ __forceinline__ float2 block_quotient(float2 a, const Bf16Block& b) {
  const float2 y = make_float2(b.inv, b.inv);
  if constexpr (MODE == kNV) {
    const float2 q0 = __fmul2_rn(a, y);
    const float2 r = __ffma2_rn(q0, make_float2(b.nscale, b.nscale), a);
    return __ffma2_rn(r, y, q0);
  } else {
    return __ffma2_rn(a, y, make_float2(0.0f, 0.0f));
  }
}

// The two elements of a bf16x2 word as floats.
__device__ __forceinline__ float2 bf16x2_to_float2(uint32_t w) {
  return make_float2(__uint_as_float(w << 16), __uint_as_float(w & 0xFFFF0000u));
}

// NW words (2*NW elements, NW a multiple of 4) of one fast-path block: reconstruction words
// and, with MASK, the in-range bits.
template <int MODE, bool MASK, int NW>
__device__ __forceinline__ void bf16_qdq_fast(const uint32_t* w, const Bf16Block& b, uint32_t* o, uint32_t& bits) {
  static_assert(NW % 4 == 0, "whole mask bytes");
#pragma unroll
  for (int i = 0; i < NW; ++i) {
    uint32_t h;
    if constexpr (MODE == kNV) {
      const float2 n = block_quotient<MODE>(bf16x2_to_float2(w[i]), b);
      h = e2m1x2_to_f16x2(n.x, n.y);
    } else {
      // MXFP4: magnitudes through the converter, the sign from the input's sign bit for a
      // nonzero input (a zero of either sign gives +0)
      const uint32_t aw = w[i] & 0x7FFF7FFFu;
      const uint32_t sg = w[i] & (aw + 0x7FFF7FFFu) & 0x80008000u;
      const float2 n = __fmul2_rn(bf16x2_to_float2(aw), make_float2(b.inv, b.inv));
      h = e2m1x2_to_f16x2(n.x, n.y) | sg;
    }
    const float2 c = __fmul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&h)), make_float2(b.scale, b.scale));
    o[i] = pack_bf16x2(c.x, c.y);
  }
  if constexpr (MASK) {
    bits = 0u;
#pragma unroll
    for (int g = 0; g < NW / 4; ++g) {
      uint32_t d[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) d[i] = b.limx - (w[4 * g + i] & 0x7FFF7FFFu);
      bits |= gather_half_msbs(d) << (8 * g);
    }
  }
}

// Packed nibbles (one word, even element in the low nibble) of one 8-element fast-path
// vector, plus the reconstruction when wanted.
template <int MODE>
__device__ __forceinline__ void bf16_pack_fast(const uint4& raw, const Bf16Block& b, bool want_recon, uint32_t& word,
                                               uint4& out) {
  const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
  float2 n[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) n[i] = block_quotient<MODE>(bf16x2_to_float2(w[i]), b);
  if (!want_recon) {
    word = e2m1_canonical(e2m1x8_word(n));
    return;
  }
  uint32_t h[4];
  word = e2m1_canonical(e2m1x8(n, h));
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 c = __fmul2_rn(__half22float2(*reinterpret_cast<const __half2*>(&h[i])), make_float2(b.scale, b.scale));
    o[i] = pack_bf16x2(c.x, c.y);
  }
  out = make_uint4(o[0], o[1], o[2], o[3]);
}

// Block amax (bf16 bits) over the 16 elements of this thread and its block partner lanes.
template <int MODE>
__device__ __forceinline__ uint32_t bf16x16_amax(const uint32_t* w) {
  uint32_t mw = max_u16x2(max_u16x2(max_u16x2(w[0] & 0x7FFF7FFFu, w[1] & 0x7FFF7FFFu),
                                    max_u16x2(w[2] & 0x7FFF7FFFu, w[3] & 0x7FFF7FFFu)),
                          max_u16x2(max_u16x2(w[4] & 0x7FFF7FFFu, w[5] & 0x7FFF7FFFu),
                                    max_u16x2(w[6] & 0x7FFF7FFFu, w[7] & 0x7FFF7FFFu)));
  uint32_t m16 = max(mw & 0xFFFFu, mw >> 16);
  if constexpr (MODE != kNV) m16 = max(m16, __shfl_xor_sync(0xffffffffu, m16, 1));
  return m16;
}

// The 16 BF16 elements of block v (one 32-byte load), or zeros past the end.
__device__ __forceinline__ void load_block16(const __nv_bfloat16* x, int64_t v, int64_t n16, uint32_t* w) {
  if (v < n16) {
    ld_stream256(x + v * 16, w);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = 0u;
  }
}

// ------------------------------------------------------------ NVFP4 GEMM operand block
// One 16-element block of the NVFP4 GEMM operand pass (qatf_nvfp4_operand, and the W4A4
// forward whose quantizer warps encode X inside the GEMM): E2M1 codes (8 bytes at
// codes + 8 v, even column in the low nibble), the dequantized block (deq, may be null), its
// 16 STE mask bits (mask, may be null) and its E4M3 scale byte.  The four blocks of one
// 64-column K-block sit in four consecutive lanes (lane 4j+i holds K-block kb + i of the same
// row as lane 4j, kb % 4 == 0), which gather their scale bytes into one 32-bit word; that word
// is stored in the layout of ROLE (see qatf.h), once in each of the four TMEM lane quarters.
// All 32 lanes call this; lanes with live false take part in the shuffles and store nothing.
// Codes and scales are quantize_nvfp4's (nvfp4.py:400-462), deq and mask
// _fake_quantize_nvfp4_torch's (nvfp4.py:465-501).  Returns the block's max |x| as BF16 bits
// (0 for a dead lane, whose raw words are zero), for a running maximum of the whole tensor.
template <int ROLE>
__device__ __forceinline__ uint32_t operand_block(const uint32_t* raw, const NvGlobal& g, int64_t v, uint32_t row,
                                                  uint32_t kb, uint32_t atoms_k, bool live, uint8_t* codes,
                                                  uint8_t* sf, __nv_bfloat16* deq, uint8_t* mask) {
  using VT = VecTraits<__nv_bfloat16>;
  const bool want_deq = deq != nullptr;
  const bool want_mask = mask != nullptr;
  const uint32_t m16 = bf16x16_amax<kNV>(raw);
  const Fp4Block p = fp4_block_bf16<kNV>(m16 << 16, g);
  uint32_t words[2] = {0u, 0u};
  uint32_t o[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
  uint32_t bits = 0xFFFFu;  // zero amax: zero codes and deq, all-true mask (nvfp4.py:427-435, :493-494)
  bool done = p.zero;
  if (!done) {
    const Bf16Block b = bf16_block<kNV>(m16, p);
    if (b.fast) {
      uint4 r0, r1;
      bf16_pack_fast<kNV>(make_uint4(raw[0], raw[1], raw[2], raw[3]), b, want_deq, words[0], r0);
      bf16_pack_fast<kNV>(make_uint4(raw[4], raw[5], raw[6], raw[7]), b, want_deq, words[1], r1);
      done = true;
      o[0] = r0.x; o[1] = r0.y; o[2] = r0.z; o[3] = r0.w;
      o[4] = r1.x; o[5] = r1.y; o[6] = r1.z; o[7] = r1.w;
      if (want_mask) {
        uint32_t d[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) d[i] = b.limx - (raw[i] & 0x7FFF7FFFu);
        bits = gather_half_msbs(d) | (gather_half_msbs(d + 4) << 8);
      }
    }
  }
  if (!done) {
    bits = 0u;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float f[8], out[8];
      VT::to_float(make_uint4(raw[4 * h], raw[4 * h + 1], raw[4 * h + 2], raw[4 * h + 3]), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float c = fp4_code<kNV>(p, f[i]);
        words[h] |= fp4_nibble(c) << (4 * i);
        out[i] = __fmul_rn(c, p.scale);
        bits |= (fabsf(f[i]) <= p.lim ? 1u : 0u) << (8 * h + i);
      }
      const uint4 q = VT::from_float(out);
      o[4 * h] = q.x;
      o[4 * h + 1] = q.y;
      o[4 * h + 2] = q.z;
      o[4 * h + 3] = q.w;
    }
  }
  // every lane of the K-block gathers the whole word, and lane 4j + q stores the copy for TMEM
  // lane quarter q (one store per lane instead of four on one lane)
  const uint32_t sbyte = p.zero ? 1u : p.byte;
  const int first = (threadIdx.x & 31) & ~3;
  const uint32_t sword = __shfl_sync(0xffffffffu, sbyte, first) | (__shfl_sync(0xffffffffu, sbyte, first + 1) << 8) |
                         (__shfl_sync(0xffffffffu, sbyte, first + 2) << 16) |
                         (__shfl_sync(0xffffffffu, sbyte, first + 3) << 24);
  if (live) {
    reinterpret_cast<uint2*>(codes)[v] = make_uint2(words[0], words[1]);
    if (want_deq) st256(deq + v * 16, o);
    if (want_mask) reinterpret_cast<uint16_t*>(mask)[v] = (uint16_t)bits;
    uint64_t blk;
    uint32_t word;
    if constexpr (ROLE == QATF_OPERAND_A) {
      blk = ((uint64_t)(row >> 7) * (atoms_k >> 1) + (kb >> 3)) * 4096u;  // 128 rows x 2 K-blocks
      word = ((kb >> 2) & 1u) * 4u + ((row >> 5) & 3u);
    } else {
      blk = ((uint64_t)(row >> 8) * atoms_k + (kb >> 2)) * 4096u;  // 256 rows x 1 K-block
      word = (row >> 5) & 7u;
    }
    const uint32_t L = (row & 31u) + 32u * (kb & 3u);  // kb % 4 == lane % 4: the lane quarter it fills
    *reinterpret_cast<uint32_t*>(sf + blk + (L >> 3) * 256u + (L & 7u) * 16u + (word >> 2) * 128u +
                                 (word & 3u) * 4u) = sword;
  }
  return m16;
}

}  // namespace qatf
