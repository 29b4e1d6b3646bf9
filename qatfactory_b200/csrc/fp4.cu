// NVFP4 / MXFP4 fake quantization, packing, dequantization, STE backward and tensor amax
// for sm_100a.
//
// Data layout: the hot kernels treat a dense [rows, cols] tensor whose rows are a whole
// number of quantization blocks (cols % 16 for NVFP4, % 32 for MXFP4) as one flat array;
// a block never straddles a row.  BF16 tensors with 32-byte aligned buffers take the
// block-per-thread kernels: one thread owns one NVFP4 block (one 32-byte load) or one MXFP4
// block (two), takes its amax as a packed 16-bit integer max over |x| bits with no shuffle,
// and (NVFP4 QDQ, packing) loads its next block before encoding the current one.  Other
// dtypes use 16-byte vectors with a block spread over 2 or 4 consecutive lanes (amax by warp
// shuffles).  Grids are one wave of resident CTAs with a grid-stride loop.  Shapes that break
// these rules (padding blocks, strided rows, unaligned pointers) take a per-element generic
// kernel with the same math.
#include "qatf.h"
#include "qatf_common.cuh"
#include "qatf_fp4.cuh"

#include <algorithm>
#include <type_traits>

namespace qatf {

// Resident CTAs per SM of the MXFP4 block-per-thread kernel.
#ifndef QATF_MX32_CTAS
#define QATF_MX32_CTAS 2
#endif
// Minimum resident CTAs per SM the BF16 pack kernel is compiled for (caps its registers):
// NVFP4 packs faster at three (configuration-4 activations 37.4 -> 35.7 us, with the
// reconstruction 58.2 -> 53.1 us), MXFP4 at four (the weight: 45.2 us against 49.7 at three).
template <int MODE>
constexpr int kPackCtas = MODE == 0 ? 3 : 4;
// Resident CTAs per SM of the BF16 NVFP4 block-per-thread kernel (0: as many as fit).
#ifndef QATF_NVW_CTAS
#define QATF_NVW_CTAS 0
#endif

constexpr int kThreads = 256;
constexpr int kUnroll = 4;


// One 32-element MXFP4 block (16 BF16 words) of the fake-quant kernel: reconstruction words
// and the block's 32 in-range bits.
template <int MODE, bool MASK>
__device__ __forceinline__ void mx32_block(const uint32_t* raw, const NvGlobal& g, uint32_t* o, uint32_t& bits) {
  using VT = VecTraits<__nv_bfloat16>;
  uint32_t mw = 0u;
#pragma unroll
  for (int i = 0; i < 16; ++i) mw = max_u16x2(mw, raw[i] & 0x7FFF7FFFu);
  const uint32_t m16 = max(mw & 0xFFFFu, mw >> 16);
  const Fp4Block p = fp4_block_bf16<MODE>(m16 << 16, g);
  bits = 0u;
  const Bf16Block bb = bf16_block<MODE>(m16, p);
  if (bb.fast) {
    uint32_t lo = 0u, hi = 0u;
    bf16_qdq_fast<MODE, MASK, 8>(raw, bb, o, lo);
    bf16_qdq_fast<MODE, MASK, 8>(raw + 8, bb, o + 8, hi);
    bits = lo | (hi << 16);
    return;
  }
#pragma unroll
  for (int h = 0; h < 4; ++h) {
    float f[8], out[8];
    VT::to_float(make_uint4(raw[4 * h], raw[4 * h + 1], raw[4 * h + 2], raw[4 * h + 3]), f);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      out[i] = p.zero ? 0.0f : __fmul_rn(fp4_code<MODE>(p, f[i]), p.scale);
      if (MASK) bits |= ((p.zero || fabsf(f[i]) <= p.lim) ? 1u : 0u) << (8 * h + i);
    }
    const uint4 q = VT::from_float(out);
    o[4 * h] = q.x;
    o[4 * h + 1] = q.y;
    o[4 * h + 2] = q.z;
    o[4 * h + 3] = q.w;
  }
}

// MXFP4 with one thread per 32-element block (64 bytes: two 32-byte loads): the block amax is a
// packed 16-bit max inside the thread, the E8M0 scale and fast-path parameters are computed
// once per block instead of once per 8 elements, and the block's 32 mask bits are one word.
// Each thread loads its next block before encoding the current one, at two CTAs per SM (the
// second block's registers leave room for no more): 67.7 us on the configuration-2 weight,
// against 71.8 us for one block in flight at three CTAs per SM, 75.5 us for the pipelined
// form squeezed into three CTAs per SM, 74.0 us for the four-lanes-per-block vector kernel
// and 79 us for a block per lane pair.
template <int MODE, bool MASK>
__global__ void __launch_bounds__(kThreads, QATF_MX32_CTAS) fp4_qdq_mx32_kernel(const __nv_bfloat16* __restrict__ x,
                                                                               __nv_bfloat16* __restrict__ y,
                                                                               uint32_t* __restrict__ mask,
                                                                               int64_t n32) {
  static_assert(MODE != kNV, "MXFP4 blocks only");
  pdl_wait();
  pdl_launch_dependents();
  const NvGlobal g = load_global<MODE>(nullptr);
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  int64_t b = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t cur[16];
  if (b < n32) {
    ld_stream256(x + b * 32, cur);
    ld_stream256(x + b * 32 + 16, cur + 8);
  }
  for (; b < n32; b += nthreads) {
    uint32_t nxt[16];
    if (b + nthreads < n32) {
      ld_stream256(x + (b + nthreads) * 32, nxt);
      ld_stream256(x + (b + nthreads) * 32 + 16, nxt + 8);
    }
    uint32_t o[16], bits;
    mx32_block<MODE, MASK>(cur, g, o, bits);
    st256(y + b * 32, o);
    st256(y + b * 32 + 16, o + 8);
    if constexpr (MASK) mask[b] = bits;
#pragma unroll
    for (int i = 0; i < 16; ++i) cur[i] = nxt[i];
  }
}

// --------------------------------------------------------------------- QDQ (vector)
template <typename T, int MODE, bool MASK>
__global__ void __launch_bounds__(kThreads) fp4_qdq_vec_kernel(const T* __restrict__ x, T* __restrict__ y,
                                                               uint8_t* __restrict__ mask, int64_t n_vec,
                                                               const float* __restrict__ tensor_amax) {
  using VT = VecTraits<T>;
  constexpr int VEC = VT::kVec;
  constexpr int LPB = Fp4Consts<MODE>::kBlock / VEC;
  const NvGlobal g = load_global<MODE>(tensor_amax);
  const int lane = threadIdx.x & 31;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t w0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); w0 < n_vec; w0 += nthreads * kUnroll) {
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = w0 + u * nthreads + lane;
      raw[u] = v < n_vec ? ld_stream(x + v * VEC) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = w0 + u * nthreads + lane;
      uint32_t m = 0u;
      uint4 packed_out;
      uint32_t bits = 0u;
      bool done = false;
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const uint32_t mw = max_u16x2(max_u16x2(raw[u].x & 0x7FFF7FFFu, raw[u].y & 0x7FFF7FFFu),
                                      max_u16x2(raw[u].z & 0x7FFF7FFFu, raw[u].w & 0x7FFF7FFFu));
        uint32_t m16 = max(mw & 0xFFFFu, mw >> 16);
#pragma unroll
        for (int o = 1; o < LPB; o <<= 1) m16 = max(m16, __shfl_xor_sync(0xffffffffu, m16, o));
        m = m16 << 16;
        const Fp4Block p = fp4_block_bf16<MODE>(m, g);
        if (p.zero && MODE == kNV) {
          packed_out = make_uint4(0u, 0u, 0u, 0u);
          bits = 0xFFu;  // NVFP4 zero amax: zeros and an all-true mask (nvfp4.py:493-494)
          done = true;
        } else {
          const Bf16Block b = bf16_block<MODE>(m16, p);
          if (b.fast) {
            const uint32_t wv[4] = {raw[u].x, raw[u].y, raw[u].z, raw[u].w};
            uint32_t ov[4];
            bf16_qdq_fast<MODE, MASK, 4>(wv, b, ov, bits);
            packed_out = make_uint4(ov[0], ov[1], ov[2], ov[3]);
            done = true;
          }
        }
        if (!done) {
          float f[VEC], out[VEC];
          VT::to_float(raw[u], f);
          if (p.zero) {
#pragma unroll
            for (int i = 0; i < VEC; ++i) out[i] = 0.0f;
          } else {
#pragma unroll
            for (int i = 0; i < VEC; ++i) {
              out[i] = __fmul_rn(fp4_code<MODE>(p, f[i]), p.scale);
              if (MASK) bits |= (fabsf(f[i]) <= p.lim ? 1u : 0u) << i;
            }
          }
          packed_out = VT::from_float(out);
        }
      } else {
        float f[VEC];
        VT::to_float(raw[u], f);
#pragma unroll
        for (int i = 0; i < VEC; ++i) m = max(m, abs_bits(f[i]));
#pragma unroll
        for (int o = 1; o < LPB; o <<= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
        const Fp4Block p = fp4_block<MODE>(m, g);
        float out[VEC];
        if (p.zero) {
#pragma unroll
          for (int i = 0; i < VEC; ++i) out[i] = 0.0f;
          bits = (1u << VEC) - 1u;  // NVFP4 zero amax: all-true mask (nvfp4.py:493-494)
        } else {
#pragma unroll
          for (int i = 0; i < VEC; ++i) {
            out[i] = __fmul_rn(fp4_code<MODE>(p, f[i]), p.scale);
            if (MASK) bits |= (fabsf(f[i]) <= p.lim ? 1u : 0u) << i;
          }
        }
        packed_out = VT::from_float(out);
      }
      if constexpr (MASK && VEC == 4) {
        const uint32_t hi = __shfl_down_sync(0xffffffffu, bits, 1);
        bits |= hi << 4;
      }
      if (v < n_vec) {
        st_v4(y + v * VEC, packed_out);
        if constexpr (MASK) {
          if constexpr (VEC == 8) {
            mask[v] = (uint8_t)bits;
          } else {
            if ((lane & 1) == 0) mask[v >> 1] = (uint8_t)bits;
          }
        }
      }
    }
  }
}


// ------------------------------------------------------- bf16 QDQ / pack, 32 B per thread
// BF16 tensors with 32-byte aligned buffers move 16 elements per thread per slot with one
// 256-bit load and one 256-bit store: an NVFP4 block is then one thread (no shuffle) and an
// MXFP4 block two lanes, which halves the per-element cost of the block scales.


// One 16-element block of the BF16 QDQ kernel: reconstruction words and mask bits.
// NVFP4 blocks first try the CTA's scale table (t, may be null); the blocks it declines, and
// MXFP4, compute their parameters per block.
template <int MODE, bool MASK>
__device__ __forceinline__ void bf16w_block(const uint32_t* raw, const NvGlobal& g, const NvScaleEntry* t, uint32_t* o,
                                            uint32_t& bits) {
  using VT = VecTraits<__nv_bfloat16>;
  const uint32_t m16 = bf16x16_amax<MODE>(raw);
  bits = 0u;
  if constexpr (MODE == kNV) {
    Bf16Block tb;
    uint32_t byte;
    if (t != nullptr && nv_block_table(m16, g, t, tb, byte)) {
      bf16_qdq_fast<MODE, MASK, 8>(raw, tb, o, bits);
      return;
    }
  }
  const Fp4Block p = fp4_block_bf16<MODE>(m16 << 16, g);
  bool done = false;
  if (MODE == kNV && p.zero) {
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = 0u;
    bits = 0xFFFFu;  // NVFP4 zero amax: zeros and an all-true mask (nvfp4.py:493-494)
    done = true;
  } else {
    const Bf16Block b = bf16_block<MODE>(m16, p);
    if (b.fast) {
      bf16_qdq_fast<MODE, MASK, 8>(raw, b, o, bits);
      done = true;
    }
  }
  if (!done) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float f[8], out[8];
      VT::to_float(make_uint4(raw[4 * h], raw[4 * h + 1], raw[4 * h + 2], raw[4 * h + 3]), f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        out[i] = p.zero ? 0.0f : __fmul_rn(fp4_code<MODE>(p, f[i]), p.scale);
        if (MASK) bits |= ((p.zero || fabsf(f[i]) <= p.lim) ? 1u : 0u) << (8 * h + i);
      }
      const uint4 q = VT::from_float(out);
      o[4 * h] = q.x;
      o[4 * h + 1] = q.y;
      o[4 * h + 2] = q.z;
      o[4 * h + 3] = q.w;
    }
  }
}

// Four CTAs per SM (at most 64 registers a thread): more warps to hide the load latency
// measured 8% faster than the unconstrained 80-register build at configuration-4 size.  Each
// thread takes one block per pass and loads the next pass's 32 bytes before computing the
// current block, so a load is in flight while it computes (configuration 1: 16.5 -> 14.5 us).
// gridDim.y > 1 batches independent tensors of n16 blocks each (the experts of a fused MoE
// weight): slice blockIdx.y starts n16 blocks further and reads its own tensor_amax entry.
template <int MODE, bool MASK>
__global__ void __launch_bounds__(kThreads, 4) fp4_qdq_bf16w_kernel(const __nv_bfloat16* __restrict__ x,
                                                                 __nv_bfloat16* __restrict__ y,
                                                                 uint8_t* __restrict__ mask, int64_t n16,
                                                                 const float* __restrict__ tensor_amax) {
  pdl_wait();
  pdl_launch_dependents();
  if (gridDim.y > 1) {
    const int64_t slice = blockIdx.y;
    x += slice * n16 * 16;
    y += slice * n16 * 16;
    if constexpr (MASK) mask += slice * n16 * 2;
    if constexpr (MODE == kNV) tensor_amax += slice;
  }
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31;
  int64_t w0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31);  // warp-uniform
  uint32_t cur[8];
  load_block16(x, w0 + lane, n16, cur);  // first, so the table is built under its latency
  const NvGlobal g = load_global<MODE>(tensor_amax);
  __shared__ NvScaleEntry table[MODE == kNV ? kNvTableEntries : 1];
  if constexpr (MODE == kNV) nv_table_build(table, g);
  for (; w0 < n16; w0 += nthreads) {
    uint32_t nxt[8];
    load_block16(x, w0 + nthreads + lane, n16, nxt);
    const int64_t v = w0 + lane;
    uint32_t o[8], bits;
    bf16w_block<MODE, MASK>(cur, g, MODE == kNV ? table : nullptr, o, bits);
    if (v < n16) {
      st256(y + v * 16, o);
      if constexpr (MASK) reinterpret_cast<uint16_t*>(mask)[v] = (uint16_t)bits;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
  }
}

// NVFP4 fake quantization of an FP32 latent shard for a gather of the quantized weight (the
// FSDP2 step quantizes each rank's shard once per optimizer step instead of the gathered BF16
// weight in every forward).  The reference fake-quantizes the weight after FSDP2's cast to BF16
// (MixedPrecisionPolicy param_dtype), so each block is first rounded to BF16 (round to nearest
// even, as torch's .to(bfloat16)), then quantized exactly as fp4_qdq_bf16w_kernel does, and its
// BF16 result is written widened to FP32 (exact), with the STE mask.  One block of 16 per
// thread and pass, the next pass's 64 bytes loaded while the current block is encoded.
__global__ void __launch_bounds__(kThreads, 3) nvfp4_qdq_shadow_kernel(const float* __restrict__ x,
                                                                    float* __restrict__ y,
                                                                    uint8_t* __restrict__ mask, int64_t n16,
                                                                    const float* __restrict__ tensor_amax) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int lane = threadIdx.x & 31;
  int64_t w0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31);  // warp-uniform
  auto load = [&](int64_t v, uint32_t* w) {
    if (v < n16) {
      ld_stream256(x + v * 16, w);
      ld_stream256(x + v * 16 + 8, w + 8);
    } else {
#pragma unroll
      for (int i = 0; i < 16; ++i) w[i] = 0u;
    }
  };
  uint32_t cur[16];
  load(w0 + lane, cur);  // first, so the table is built under its latency
  const NvGlobal g = load_global<kNV>(tensor_amax);
  __shared__ NvScaleEntry table[kNvTableEntries];
  nv_table_build(table, g);
  for (; w0 < n16; w0 += nthreads) {
    uint32_t nxt[16];
    load(w0 + nthreads + lane, nxt);
    const int64_t v = w0 + lane;
    uint32_t raw[8], o[8], bits;
#pragma unroll
    for (int i = 0; i < 8; ++i) raw[i] = pack_bf16x2(__uint_as_float(cur[2 * i]), __uint_as_float(cur[2 * i + 1]));
    bf16w_block<kNV, true>(raw, g, table, o, bits);
    if (v < n16) {
      uint32_t lo[8], hi[8];  // BF16 -> FP32 is the high half of the word
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        lo[2 * i] = o[i] << 16;
        lo[2 * i + 1] = o[i] & 0xFFFF0000u;
        hi[2 * i] = o[4 + i] << 16;
        hi[2 * i + 1] = o[4 + i] & 0xFFFF0000u;
      }
      st256(y + v * 16, lo);
      st256(y + v * 16 + 8, hi);
      reinterpret_cast<uint16_t*>(mask)[v] = (uint16_t)bits;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) cur[i] = nxt[i];
  }
}

template <int MODE>
__global__ void __launch_bounds__(kThreads, kPackCtas<MODE>) fp4_pack_bf16w_kernel(const __nv_bfloat16* __restrict__ x, int64_t n16,
                                                                  const float* __restrict__ tensor_amax,
                                                                  uint8_t* __restrict__ packed,
                                                                  uint8_t* __restrict__ scales,
                                                                  float* __restrict__ scale_2,
                                                                  __nv_bfloat16* __restrict__ recon) {
  using VT = VecTraits<__nv_bfloat16>;
  pdl_wait();
  pdl_launch_dependents();
  const bool want_recon = recon != nullptr;
  const int lane = threadIdx.x & 31;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  int64_t w0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31);  // warp-uniform
  uint32_t raw[8];
  load_block16(x, w0 + lane, n16, raw);  // first, so the table is built under its latency
  const NvGlobal g = load_global<MODE>(tensor_amax);
  __shared__ NvScaleEntry table[MODE == kNV ? kNvTableEntries : 1];
  if constexpr (MODE == kNV) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_2 = g.zero ? 1.0f : g.gs;  // nvfp4.py:434, :437
    nv_table_build(table, g);
  }
  for (; w0 < n16; w0 += nthreads) {
    uint32_t nxt[8];  // the next pass's block, in flight while this one is encoded
    load_block16(x, w0 + nthreads + lane, n16, nxt);
    {
      const int64_t v = w0 + lane;
      const uint32_t m16 = bf16x16_amax<MODE>(raw);
      uint32_t words[2] = {0u, 0u};
      uint32_t o[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
      uint32_t sbyte = 0u;
      bool done = false;
      if constexpr (MODE == kNV) {
        Bf16Block tb;
        if (nv_block_table(m16, g, table, tb, sbyte)) {
          uint4 r0, r1;
          bf16_pack_fast<MODE>(make_uint4(raw[0], raw[1], raw[2], raw[3]), tb, want_recon, words[0], r0);
          bf16_pack_fast<MODE>(make_uint4(raw[4], raw[5], raw[6], raw[7]), tb, want_recon, words[1], r1);
          o[0] = r0.x; o[1] = r0.y; o[2] = r0.z; o[3] = r0.w;
          o[4] = r1.x; o[5] = r1.y; o[6] = r1.z; o[7] = r1.w;
          done = true;
        }
      }
      if (!done) {  // the table declined the block (or MXFP4): parameters per block
        const Fp4Block p = fp4_block_bf16<MODE>(m16 << 16, g);
        sbyte = p.zero ? 1u : p.byte;
        done = p.zero;  // NVFP4 zero amax: codes 0, scales 2^-9 (nvfp4.py:427-435)
        if (!done) {
          const Bf16Block b = bf16_block<MODE>(m16, p);
          if (b.fast) {
            uint4 r0, r1;
            bf16_pack_fast<MODE>(make_uint4(raw[0], raw[1], raw[2], raw[3]), b, want_recon, words[0], r0);
            bf16_pack_fast<MODE>(make_uint4(raw[4], raw[5], raw[6], raw[7]), b, want_recon, words[1], r1);
            o[0] = r0.x; o[1] = r0.y; o[2] = r0.z; o[3] = r0.w;
            o[4] = r1.x; o[5] = r1.y; o[6] = r1.z; o[7] = r1.w;
            done = true;
          }
        }
        if (!done) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            float f[8], out[8];
            VT::to_float(make_uint4(raw[4 * h], raw[4 * h + 1], raw[4 * h + 2], raw[4 * h + 3]), f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float c = fp4_code<MODE>(p, f[i]);
              words[h] |= fp4_nibble(c) << (4 * i);
              out[i] = __fmul_rn(c, p.scale);
            }
            const uint4 q = VT::from_float(out);
            o[4 * h] = q.x;
            o[4 * h + 1] = q.y;
            o[4 * h + 2] = q.z;
            o[4 * h + 3] = q.w;
          }
        }
      }
      if (v < n16) {
        reinterpret_cast<uint2*>(packed)[v] = make_uint2(words[0], words[1]);
        if (MODE == kNV || (lane & 1) == 0) scales[MODE == kNV ? v : v >> 1] = (uint8_t)sbyte;
        if (want_recon) st256(recon + v * 16, o);
      }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) raw[i] = nxt[i];
  }
}

// ------------------------------------------------------------ NVFP4 GEMM operand
// One pass over a BF16 [rows, cols] tensor producing what the W4A4 GEMMs consume: packed E2M1
// codes, E4M3 block scales in the layout of the operand's role (see qatf.h), and optionally
// the dequantized tensor and the STE mask.  A thread owns one 16-element block; the four
// blocks of one 64-column K-block are consecutive lanes, whose scale bytes are gathered into
// one 32-bit word:
//   A role: a 4 KB block per 128 rows x 128 columns (two K-blocks): lane L holds, for K-block
//           j of the block and c = 0..3, the word of row 32c + L%32 as word 4j + c;
//   B role: a 4 KB block per 256 rows x 64 columns (one K-block): lane L holds the word of row
//           32h + L%32 as word h, h = 0..7.
// Either way a row's word is written to the four lanes L = r%32 + 32q of its block (the four
// TMEM lane quarters each need every scale), and one tcgen05.cp 128x256b moves a block into
// eight TMEM columns.  Blocks are core matrices of 8 lanes x 16 bytes (halves 128 bytes apart,
// 8-lane groups 256 bytes apart); word v of lane L is at (L/8)*256 + (L%8)*16 + (v/4)*128 + (v%4)*4.
// Resident CTAs per SM of the operand pass, which loads the next pass's block while it encodes
// the current one: two for the A side (X: 66.4 against 68.3 us without the pipelining), three
// for the B side (W: 27.3 against 29.0 us), measured at configuration 4.  More do not help:
// three A-side CTAs (80 registers) ran X in 67.8 us against 66.0-67.3, four (spilling) 77.7;
// four B-side CTAs ran W in 32.8 us against 28.2-29.1.
#ifndef QATF_OPERAND_A_CTAS
#define QATF_OPERAND_A_CTAS 2
#endif
#ifndef QATF_OPERAND_B_CTAS
#define QATF_OPERAND_B_CTAS 3
#endif
template <int ROLE>
constexpr int kOperandCtas = ROLE == QATF_OPERAND_A ? QATF_OPERAND_A_CTAS : QATF_OPERAND_B_CTAS;

template <int ROLE>
__global__ void __launch_bounds__(kThreads, kOperandCtas<ROLE>) nvfp4_operand_bf16_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t n16, uint32_t cols16, const float* __restrict__ tensor_amax,
    uint8_t* __restrict__ codes, uint8_t* __restrict__ sf, __nv_bfloat16* __restrict__ deq,
    uint8_t* __restrict__ mask, uint32_t* __restrict__ running_bits) {
  const uint32_t atoms_k = cols16 >> 2;
  const int lane = threadIdx.x & 31;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  int64_t w0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31);
  uint32_t raw[8];
  uint32_t seen = 0u;  // max |x| of this thread's blocks, as BF16 bits
  load_block16(x, w0 + lane, n16, raw);
  // parameters per block, not the CTA's scale table: the table measured 2% slower here (X 67.3
  // against 65.8 us), where the block's other work (scale-word gather, four outputs) dominates
  const NvGlobal g = load_global<kNV>(tensor_amax);
  // (row, column block) of this thread's block, advanced by the grid stride without a division
  // per block (n16 < 2^32, checked by the entry point)
  const uint32_t step_rows = (uint32_t)nthreads / cols16, step_cols = (uint32_t)nthreads % cols16;
  uint32_t row = (uint32_t)(w0 + lane) / cols16;
  uint32_t kb = (uint32_t)(w0 + lane) - row * cols16;
  for (; w0 < n16; w0 += nthreads) {
    uint32_t nxt[8];
    load_block16(x, w0 + nthreads + lane, n16, nxt);
    const int64_t v = w0 + lane;
    seen = max(seen, operand_block<ROLE>(raw, g, v, row, kb, atoms_k, v < n16, codes, sf, deq, mask));
    row += step_rows;
    kb += step_cols;
    if (kb >= cols16) {
      kb -= cols16;
      ++row;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) raw[i] = nxt[i];
  }
  if (running_bits != nullptr) {  // running maximum: FP32 bits of a non-negative value or NaN order as integers
    seen = __reduce_max_sync(0xffffffffu, seen);
    if (lane == 0) atomicMax(running_bits, seen << 16);
  }
}

// ------------------------------------------------------------ MXFP4 GEMM operand
// The same pass for qatf_mxfp4_gemm: E2M1 codes, E8M0 block-32 scales (EVEN rule for weights,
// CEIL for activations, mxfp4.py:48-98) in the layout of the operand's role, and optionally
// the dequantized tensor and the STE mask (all true under CEIL, whose STE is unmasked).  Two
// lanes share a 32-element block (16 elements each; the block amax takes one shuffle, as in
// the MXFP4 QDQ and pack kernels), so the eight lanes of a 128-column K-block hold its four
// scale bytes (lanes 8j, 8j + 2, 8j + 4, 8j + 6); they gather them into one 32-bit word, which
// the even lanes store into the four TMEM lane quarters.  The block-32 word spans 128 columns
// where NVFP4's spans 64, so an A block covers 128 rows x 256 columns and a B block 256 rows x
// 128 columns.
template <int ROLE, int MODE>
__global__ void __launch_bounds__(kThreads, 3) mxfp4_operand_bf16_kernel(
    const __nv_bfloat16* __restrict__ x, int64_t n16, uint32_t cols16, uint8_t* __restrict__ codes,
    uint8_t* __restrict__ sf, __nv_bfloat16* __restrict__ deq, uint8_t* __restrict__ mask) {
  using VT = VecTraits<__nv_bfloat16>;
  pdl_wait();
  pdl_launch_dependents();
  const NvGlobal g = load_global<MODE>(nullptr);  // MXFP4 has no tensor scale
  const bool want_deq = deq != nullptr;
  const bool want_mask = mask != nullptr;
  const uint32_t kblocks = cols16 >> 3;  // 128-column K-blocks per row
  const int lane = threadIdx.x & 31;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  int64_t w0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31);
  uint32_t raw[8];
  load_block16(x, w0 + lane, n16, raw);
  // (row, 16-column chunk) of this thread, advanced by the grid stride (n16 < 2^32)
  const uint32_t step_rows = (uint32_t)nthreads / cols16, step_cols = (uint32_t)nthreads % cols16;
  uint32_t row = (uint32_t)(w0 + lane) / cols16;
  uint32_t c16 = (uint32_t)(w0 + lane) - row * cols16;
  for (; w0 < n16; w0 += nthreads) {
    uint32_t nxt[8];
    load_block16(x, w0 + nthreads + lane, n16, nxt);
    const int64_t v = w0 + lane;
    const uint32_t m16 = bf16x16_amax<MODE>(raw);  // the pair's block amax (one shuffle)
    const Fp4Block p = fp4_block<MODE>(m16 << 16, g);
    uint32_t words[2] = {0u, 0u};
    uint32_t o[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    uint32_t bits = 0xFFFFu;
    bool done = p.zero;  // CEIL zero block: zero codes and deq (mxfp4.py:96-98)
    if (!done) {
      const Bf16Block b = bf16_block<MODE>(m16, p);
      if (b.fast) {
        uint4 r0, r1;
        bf16_pack_fast<MODE>(make_uint4(raw[0], raw[1], raw[2], raw[3]), b, want_deq, words[0], r0);
        bf16_pack_fast<MODE>(make_uint4(raw[4], raw[5], raw[6], raw[7]), b, want_deq, words[1], r1);
        o[0] = r0.x; o[1] = r0.y; o[2] = r0.z; o[3] = r0.w;
        o[4] = r1.x; o[5] = r1.y; o[6] = r1.z; o[7] = r1.w;
        if (want_mask) {
          uint32_t d[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) d[i] = b.limx - (raw[i] & 0x7FFF7FFFu);
          bits = gather_half_msbs(d) | (gather_half_msbs(d + 4) << 8);
        }
        done = true;
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
          const float c = fp4_code<MODE>(p, f[i]);
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
    const int first = lane & ~7;
    const uint32_t sword = __shfl_sync(0xffffffffu, p.byte, first) | (__shfl_sync(0xffffffffu, p.byte, first + 2) << 8) |
                           (__shfl_sync(0xffffffffu, p.byte, first + 4) << 16) |
                           (__shfl_sync(0xffffffffu, p.byte, first + 6) << 24);
    if (v < n16) {
      reinterpret_cast<uint2*>(codes)[v] = make_uint2(words[0], words[1]);
      if (want_deq) st256(deq + v * 16, o);
      if (want_mask) reinterpret_cast<uint16_t*>(mask)[v] = (uint16_t)bits;
      if ((lane & 1) == 0) {
        const uint32_t kb = c16 >> 3;
        uint64_t blk;
        uint32_t word;
        if constexpr (ROLE == QATF_OPERAND_A) {
          blk = ((uint64_t)(row >> 7) * (kblocks >> 1) + (kb >> 1)) * 4096u;  // 128 rows x 2 K-blocks
          word = (kb & 1u) * 4u + ((row >> 5) & 3u);
        } else {
          blk = ((uint64_t)(row >> 8) * kblocks + kb) * 4096u;  // 256 rows x 1 K-block
          word = (row >> 5) & 7u;
        }
        const uint32_t L = (row & 31u) + 32u * (((uint32_t)lane >> 1) & 3u);  // lane quarter (lane / 2) % 4
        *reinterpret_cast<uint32_t*>(sf + blk + (L >> 3) * 256u + (L & 7u) * 16u + (word >> 2) * 128u +
                                     (word & 3u) * 4u) = sword;
      }
    }
    row += step_rows;
    c16 += step_cols;
    if (c16 >= cols16) {
      c16 -= cols16;
      ++row;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) raw[i] = nxt[i];
  }
}

// -------------------------------------------------------------------- QDQ (generic)
// One thread per mask byte (8 flat elements); block scales are recomputed per block.
template <typename T, int MODE, bool MASK>
__global__ void __launch_bounds__(kThreads) fp4_qdq_generic_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                                                   int64_t ld, T* __restrict__ y,
                                                                   uint8_t* __restrict__ mask,
                                                                   const float* __restrict__ tensor_amax) {
  using VT = VecTraits<T>;
  constexpr int B = Fp4Consts<MODE>::kBlock;
  const NvGlobal g = load_global<MODE>(tensor_amax);
  const int64_t n = rows * cols;
  const int64_t n_groups = (n + 7) / 8;
  for (int64_t grp = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; grp < n_groups;
       grp += (int64_t)gridDim.x * blockDim.x) {
    uint32_t bits = 0u;
    int64_t cached = -1;
    Fp4Block p;
    for (int i = 0; i < 8; ++i) {
      const int64_t e = grp * 8 + i;
      if (e >= n) break;
      const int64_t r = e / cols, c = e - r * cols;
      const int64_t c0 = (c / B) * B;
      const int64_t key = r * cols + c0;
      if (key != cached) {
        uint32_t m = 0u;
        const int64_t c1 = c0 + B < cols ? c0 + B : cols;
        for (int64_t k = c0; k < c1; ++k) m = max(m, abs_bits(VT::load1(x + r * ld + k)));
        p = fp4_block<MODE>(m, g);
        cached = key;
      }
      const float v = VT::load1(x + r * ld + c);
      float out = 0.0f;
      bool in_range = true;
      if (!p.zero) {
        out = __fmul_rn(fp4_code<MODE>(p, v), p.scale);
        in_range = fabsf(v) <= p.lim;
      }
      VT::store1(y + e, out);
      bits |= (in_range ? 1u : 0u) << i;
    }
    if (MASK) mask[grp] = (uint8_t)bits;
  }
}

// ------------------------------------------------------------------------- packing
// Vector pack for dense, 16-byte aligned inputs with cols % block == 0.  Each thread emits
// VEC/2 packed bytes; the first lane of each block writes the block's scale byte.
template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads) fp4_pack_vec_kernel(const T* __restrict__ x, int64_t n_vec,
                                                                const float* __restrict__ tensor_amax,
                                                                uint8_t* __restrict__ packed,
                                                                uint8_t* __restrict__ scales,
                                                                float* __restrict__ scale_2, T* __restrict__ recon) {
  using VT = VecTraits<T>;
  constexpr int VEC = VT::kVec;
  constexpr int LPB = Fp4Consts<MODE>::kBlock / VEC;
  const NvGlobal g = load_global<MODE>(tensor_amax);
  if constexpr (MODE == kNV) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_2 = g.zero ? 1.0f : g.gs;  // nvfp4.py:434, :437
  }
  const int lane = threadIdx.x & 31;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t w0 = (int64_t)blockIdx.x * blockDim.x + (threadIdx.x & ~31); w0 < n_vec; w0 += nthreads * kUnroll) {
    uint4 raw[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = w0 + u * nthreads + lane;
      raw[u] = v < n_vec ? ld_stream(x + v * VEC) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int64_t v = w0 + u * nthreads + lane;
      uint32_t word = 0u;
      uint4 rc = make_uint4(0u, 0u, 0u, 0u);
      uint32_t scale_byte;
      bool done = false;
      uint32_t m = 0u;
      if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const uint32_t mw = max_u16x2(max_u16x2(raw[u].x & 0x7FFF7FFFu, raw[u].y & 0x7FFF7FFFu),
                                      max_u16x2(raw[u].z & 0x7FFF7FFFu, raw[u].w & 0x7FFF7FFFu));
        uint32_t m16 = max(mw & 0xFFFFu, mw >> 16);
#pragma unroll
        for (int o = 1; o < LPB; o <<= 1) m16 = max(m16, __shfl_xor_sync(0xffffffffu, m16, o));
        m = m16 << 16;
      } else {
        float f[VEC];
        VT::to_float(raw[u], f);
#pragma unroll
        for (int i = 0; i < VEC; ++i) m = max(m, abs_bits(f[i]));
#pragma unroll
        for (int o = 1; o < LPB; o <<= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
      }
      const Fp4Block p = std::is_same<T, __nv_bfloat16>::value ? fp4_block_bf16<MODE>(m, g) : fp4_block<MODE>(m, g);
      scale_byte = p.zero ? 1u : p.byte;
      if (p.zero) {  // NVFP4 zero amax: codes 0, scales 2^-9 (nvfp4.py:427-435)
        done = true;
      } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
        const Bf16Block b = bf16_block<MODE>(m >> 16, p);
        if (b.fast) {
          bf16_pack_fast<MODE>(raw[u], b, recon != nullptr, word, rc);
          done = true;
        }
      }
      if (!done) {
        float f[VEC], out[VEC];
        VT::to_float(raw[u], f);
#pragma unroll
        for (int i = 0; i < VEC; ++i) {
          const float c = fp4_code<MODE>(p, f[i]);
          word |= fp4_nibble(c) << (4 * i);
          out[i] = __fmul_rn(c, p.scale);
        }
        rc = VT::from_float(out);
      }
      if (v < n_vec) {
        if constexpr (VEC == 8) {
          reinterpret_cast<uint32_t*>(packed)[v] = word;
        } else {
          reinterpret_cast<uint16_t*>(packed)[v] = (uint16_t)word;
        }
        if (lane % LPB == 0) scales[v / LPB] = (uint8_t)scale_byte;
        if (recon != nullptr) st_v4(recon + v * VEC, rc);
      }
    }
  }
}

// Generic pack: one thread per packed byte (two elements), any row stride / alignment.
template <typename T, int MODE>
__global__ void __launch_bounds__(kThreads) fp4_pack_generic_kernel(const T* __restrict__ x, int64_t rows,
                                                                    int64_t cols, int64_t ld,
                                                                    const float* __restrict__ tensor_amax,
                                                                    uint8_t* __restrict__ packed,
                                                                    uint8_t* __restrict__ scales,
                                                                    float* __restrict__ scale_2,
                                                                    T* __restrict__ recon) {
  using VT = VecTraits<T>;
  constexpr int B = Fp4Consts<MODE>::kBlock;
  const NvGlobal g = load_global<MODE>(tensor_amax);
  if constexpr (MODE == kNV) {
    if (blockIdx.x == 0 && threadIdx.x == 0) *scale_2 = g.zero ? 1.0f : g.gs;
  }
  const int64_t n_pairs = rows * cols / 2;
  for (int64_t pi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; pi < n_pairs;
       pi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = pi * 2;
    const int64_t r = e / cols, c = e - r * cols;
    const int64_t c0 = (c / B) * B;
    uint32_t m = 0u;
    for (int k = 0; k < B; ++k) m = max(m, abs_bits(VT::load1(x + r * ld + c0 + k)));
    const Fp4Block p = fp4_block<MODE>(m, g);
    uint32_t byte = 0u;
    for (int h = 0; h < 2; ++h) {
      const float v = VT::load1(x + r * ld + c + h);
      float out = 0.0f;
      if (!p.zero) {
        const float code = fp4_code<MODE>(p, v);
        byte |= fp4_nibble(code) << (4 * h);
        out = __fmul_rn(code, p.scale);
      }
      if (recon != nullptr) VT::store1(recon + e + h, out);
    }
    packed[pi] = (uint8_t)byte;
    if (c == c0) scales[r * (cols / B) + c / B] = (uint8_t)(p.zero ? 1u : p.byte);
  }
}

// ---------------------------------------------------------------------- dequantize
__device__ __forceinline__ float e2m1_value(uint32_t nib) {
  const float mag = nib & 4u ? ((nib & 3u) == 0u ? 2.0f : ((nib & 3u) == 1u ? 3.0f : ((nib & 3u) == 2u ? 4.0f : 6.0f)))
                             : __fmul_rn((float)(nib & 3u), 0.5f);
  return (nib & 8u) ? -mag : mag;
}

__device__ __forceinline__ float e4m3_value(uint32_t byte) {
  const uint32_t e = (byte >> 3) & 0xFu, m = byte & 7u;
  if (e == 0xFu && m == 7u) return __int_as_float(0x7FC00000);
  if (e == 0u) return __fmul_rn((float)m, 0.001953125f);
  return __uint_as_float(((e + 120u) << 23) | (m << 20));
}

// NVFP4: out = level * (E4M3 scale * scale_2) (nvfp4.py:111-121).  One thread per packed byte.
__global__ void __launch_bounds__(kThreads) nvfp4_dequant_kernel(const uint8_t* __restrict__ packed,
                                                                 const uint8_t* __restrict__ scales,
                                                                 const float* __restrict__ scale_2, int64_t rows,
                                                                 int64_t cols, float* __restrict__ out) {
  const float s2 = __ldg(scale_2);
  const int64_t n_pairs = rows * cols / 2;
  for (int64_t pi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; pi < n_pairs;
       pi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = pi * 2;
    const int64_t r = e / cols, c = e - r * cols;
    const float eff = __fmul_rn(e4m3_value(scales[r * (cols / 16) + c / 16]), s2);
    const uint32_t b = packed[pi];
    float2 o;
    o.x = __fmul_rn(e2m1_value(b & 0xFu), eff);
    o.y = __fmul_rn(e2m1_value(b >> 4), eff);
    reinterpret_cast<float2*>(out)[pi] = o;
  }
}

// MXFP4: out = level * 2^(byte - 127) (mxfp4.py:106-116).
__global__ void __launch_bounds__(kThreads) mxfp4_dequant_kernel(const uint8_t* __restrict__ packed,
                                                                 const uint8_t* __restrict__ scales, int64_t rows,
                                                                 int64_t cols, float* __restrict__ out) {
  const int64_t n_pairs = rows * cols / 2;
  for (int64_t pi = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; pi < n_pairs;
       pi += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = pi * 2;
    const int64_t r = e / cols, c = e - r * cols;
    const float s = pow2i((int)scales[r * (cols / 32) + c / 32] - 127);
    const uint32_t b = packed[pi];
    float2 o;
    o.x = __fmul_rn(e2m1_value(b & 0xFu), s);
    o.y = __fmul_rn(e2m1_value(b >> 4), s);
    reinterpret_cast<float2*>(out)[pi] = o;
  }
}

// Vectorised dequantization of a dense tensor: thread f writes the float4 of elements 4f..4f+3
// (consecutive threads write consecutive 16-byte chunks), reading their two code bytes
// (bytes 2f, 2f+1 of `packed`) and their block's scale byte (byte 4f / B of `scales`).  Codes
// are expanded by the hardware E2M1 -> f16 converter (exact; nibble 8 gives -0 like the
// reference's where(sign, -level, level)); one FP32 multiply per element.
__device__ __forceinline__ float4 e2m1x4_scaled(uint32_t two_bytes, float eff) {
  uint32_t h0, h1;
  asm("{\n\t.reg .b8 t;\n\tmov.b32 {t, _, _, _}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(h0) : "r"(two_bytes));
  asm("{\n\t.reg .b8 t;\n\tmov.b32 {t, _, _, _}, %1;\n\tcvt.rn.f16x2.e2m1x2 %0, t;\n\t}" : "=r"(h1) : "r"(two_bytes >> 8));
  const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&h0));
  const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&h1));
  return make_float4(__fmul_rn(a.x, eff), __fmul_rn(a.y, eff), __fmul_rn(b.x, eff), __fmul_rn(b.y, eff));
}

template <int MODE>
__global__ void __launch_bounds__(kThreads) fp4_dequant_vec_kernel(const uint16_t* __restrict__ packed2,
                                                                   const uint8_t* __restrict__ scales,
                                                                   const float* __restrict__ scale_2, int64_t n4,
                                                                   float4* __restrict__ out) {
  constexpr int B = Fp4Consts<MODE>::kBlock;
  constexpr int U = 4;
  const float s2 = MODE == kNV ? __ldg(scale_2) : 1.0f;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t f0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; f0 < n4; f0 += nthreads * U) {
    uint32_t c[U], sb[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t f = f0 + u * nthreads;
      c[u] = f < n4 ? (uint32_t)__ldg(packed2 + f) : 0u;
      sb[u] = f < n4 ? (uint32_t)__ldg(scales + (f * 4) / B) : 0u;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t f = f0 + u * nthreads;
      const float eff = MODE == kNV ? __fmul_rn(e4m3_value(sb[u]), s2) : pow2i((int)sb[u] - 127);
      if (f < n4) out[f] = e2m1x4_scaled(c[u], eff);
    }
  }
}

// ------------------------------------------------------------------- STE backward
// grad_in = grad_out * in_range, evaluated as an FP32 multiply by 1 or 0 and rounded back
// (exact: g * 1 == g; g * 0 == +-0, or NaN for inf/NaN g) like torch's bf16 * bool.
template <typename T>
__global__ void __launch_bounds__(kThreads) ste_vec_kernel(const T* __restrict__ g, const uint8_t* __restrict__ mask,
                                                           T* __restrict__ out, int64_t n_vec) {
  using VT = VecTraits<T>;
  constexpr int VEC = VT::kVec;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < n_vec; v += nthreads) {
    float f[VEC];
    VT::to_float(ld_stream(g + v * VEC), f);
    uint32_t bits = mask[(v * VEC) >> 3];
    if constexpr (VEC == 4) bits >>= (v & 1) * 4;
#pragma unroll
    for (int i = 0; i < VEC; ++i) f[i] = __fmul_rn(f[i], (bits >> i) & 1u ? 1.0f : 0.0f);
    st_v4(out + v * VEC, VT::from_float(f));
  }
}

// BF16 with 32-byte aligned buffers: 16 elements (one 32-byte load, two mask bytes) per thread
// and pass, the next pass's gradient loaded before the current one is masked, with the same
// FP32 multiply by 1 or 0 as the vector kernel.
__global__ void __launch_bounds__(kThreads) ste_bf16w_kernel(const __nv_bfloat16* __restrict__ g,
                                                             const uint16_t* __restrict__ mask16,
                                                             __nv_bfloat16* __restrict__ out, int64_t n16) {
  pdl_wait();
  pdl_launch_dependents();
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t cur[8];
  if (v < n16) ld_stream256(g + v * 16, cur);
  for (; v < n16; v += nthreads) {
    uint32_t nxt[8];
    if (v + nthreads < n16) ld_stream256(g + (v + nthreads) * 16, nxt);
    const uint32_t bits = __ldg(mask16 + v);
    uint32_t o[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float f[2];
      VecTraits<__nv_bfloat16>::unpack2(cur[i], f);
      o[i] = pack_bf16x2(__fmul_rn(f[0], (bits >> (2 * i)) & 1u ? 1.0f : 0.0f),
                         __fmul_rn(f[1], (bits >> (2 * i + 1)) & 1u ? 1.0f : 0.0f));
    }
    st256(out + v * 16, o);
#pragma unroll
    for (int i = 0; i < 8; ++i) cur[i] = nxt[i];
  }
}

template <typename T>
__global__ void __launch_bounds__(kThreads) ste_generic_kernel(const T* __restrict__ g,
                                                               const uint8_t* __restrict__ mask,
                                                               T* __restrict__ out, int64_t n) {
  using VT = VecTraits<T>;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const float m = (mask[e >> 3] >> (e & 7)) & 1u ? 1.0f : 0.0f;
    VT::store1(out + e, __fmul_rn(VT::load1(g + e), m));
  }
}

// ---------------------------------------------------------------------- tensor amax
// max |x| bits over a dense tensor.  One resident wave of 256-thread blocks, each thread with U
// 32-byte loads in flight and registers capped so that 16 / U blocks fit on an SM: U = 2 for one
// tensor, U = 4 for the batched expert form (measured: a 32 MB weight 7.4 µs at U = 2 against
// 7.9 at U = 4; 64 experts of 6 MB 71.7 µs at U = 4 against 77.6 at U = 2); BF16 magnitudes are compared as packed 16-bit integers (|x| bits order like |x|, NaN
// above inf, so NaN propagates as in torch's amax).  One atomicMax per block on the FP32 bits of
// the result.  The result is zeroed by amax_zero_kernel, launched with programmatic dependent
// launch like the reduction itself, so a chain of quantizer launches keeps overlapping one
// launch's ramp with the previous one's tail (a memset would be a plain stream-ordered node).
constexpr int kAmaxThreads = 256;

__global__ void __launch_bounds__(128) amax_zero_kernel(uint32_t* __restrict__ bits, int64_t count) {
  pdl_wait();  // the previous launch may still read the old maximum
  pdl_launch_dependents();
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < count; i += (int64_t)gridDim.x * blockDim.x)
    bits[i] = 0u;
}

template <typename T>
__device__ __forceinline__ uint32_t amax_bits32(const uint32_t* w) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) {
    uint32_t mw = 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) mw = max_u16x2(mw, w[i] & 0x7FFF7FFFu);
    return max(mw & 0xFFFFu, mw >> 16) << 16;
  } else {
    uint4 lo = make_uint4(w[0], w[1], w[2], w[3]), hi = make_uint4(w[4], w[5], w[6], w[7]);
    float f[2 * VecTraits<T>::kVec];
    VecTraits<T>::to_float(lo, f);
    VecTraits<T>::to_float(hi, f + VecTraits<T>::kVec);
    uint32_t m = 0u;
#pragma unroll
    for (int i = 0; i < 2 * VecTraits<T>::kVec; ++i) m = max(m, abs_bits(f[i]));
    return m;
  }
}

template <typename T, int kAmaxUnroll>
__global__ void __launch_bounds__(kAmaxThreads, 16 / kAmaxUnroll) amax_kernel(const T* __restrict__ x, int64_t n,
                                                                              int vec_ok, uint32_t* __restrict__ out_bits) {
  constexpr int EPC = 32 / sizeof(T);  // elements per 32-byte chunk
  pdl_wait();
  pdl_launch_dependents();
  // gridDim.y > 1: independent slices of n elements each (the experts of a fused MoE weight),
  // slice blockIdx.y reducing into out_bits[blockIdx.y]
  x += (int64_t)blockIdx.y * n;
  out_bits += blockIdx.y;
  const int64_t nthreads = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t m = 0u;
  int64_t tail = 0;
  if (vec_ok) {
    const int64_t n_chunks = n / EPC;
    // this thread's chunks are tid, tid + nthreads, ...: a pointer stepped by a fixed stride
    uint32_t count = tid < n_chunks ? (uint32_t)((n_chunks - tid + nthreads - 1) / nthreads) : 0u;
    const T* p = x + tid * EPC;
    const int64_t stride = nthreads * EPC;
    for (; count >= (uint32_t)kAmaxUnroll; count -= kAmaxUnroll) {
      uint32_t r[kAmaxUnroll][8];
#pragma unroll
      for (int u = 0; u < kAmaxUnroll; ++u) ld_stream256(p + u * stride, r[u]);
      p += kAmaxUnroll * stride;
#pragma unroll
      for (int u = 0; u < kAmaxUnroll; ++u) m = max(m, amax_bits32<T>(r[u]));
    }
    for (; count > 0u; --count, p += stride) {
      uint32_t r0[8];
      ld_stream256(p, r0);
      m = max(m, amax_bits32<T>(r0));
    }
    tail = n_chunks * EPC;
  }
  for (int64_t e = tail + tid; e < n; e += nthreads) m = max(m, abs_bits(VecTraits<T>::load1(x + e)));
  m = __reduce_max_sync(0xffffffffu, m);
  __shared__ uint32_t warp_max[kAmaxThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_max[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x < 32) {
    m = threadIdx.x < kAmaxThreads / 32 ? warp_max[threadIdx.x] : 0u;
    m = __reduce_max_sync(0xffffffffu, m);
    if (threadIdx.x == 0) atomicMax(out_bits, m);
  }
}

__global__ void e2m1_pack_rows_kernel(const uint8_t* __restrict__ nib, int64_t n_pairs, uint8_t* __restrict__ packed) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_pairs; i += (int64_t)gridDim.x * blockDim.x)
    packed[i] = (uint8_t)((nib[2 * i] & 0x0Fu) | ((nib[2 * i + 1] & 0x0Fu) << 4));
}

__global__ void e2m1_unpack_rows_kernel(const uint8_t* __restrict__ packed, int64_t n_bytes, uint8_t* __restrict__ nib) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n_bytes; i += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t b = packed[i];
    nib[2 * i] = b & 0x0Fu;
    nib[2 * i + 1] = (b >> 4) & 0x0Fu;
  }
}

// ------------------------------------------------------------------- host dispatch
inline int64_t grid_for(int64_t work_items, const void* kernel) { return persistent_grid(work_items, kernel, kThreads); }

inline int launch_status() { return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH); }

template <typename F>
int dispatch_dtype(int dtype, F&& f) {
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

template <int MODE>
int fp4_qdq(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float* tensor_amax, void* y,
            uint8_t* mask, cudaStream_t stream) {
  if (rows < 0 || cols < 0 || ld < cols || (rows > 0 && cols > 0 && (x == nullptr || y == nullptr)))
    return QATF_ERR_INVALID;
  if (MODE == kNV && tensor_amax == nullptr) return QATF_ERR_INVALID;
  if (MODE == kMXCeil && cols % 32 != 0) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  constexpr int B = Fp4Consts<MODE>::kBlock;
  return dispatch_dtype(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    const T* xt = static_cast<const T*>(x);
    T* yt = static_cast<T*>(y);
    const int64_t n = rows * cols;
    const bool vec = (cols % B == 0) && (ld == cols) && aligned16(x) && aligned16(y);
    const bool wide = std::is_same<T, __nv_bfloat16>::value && vec && aligned32(x) && aligned32(y) &&
                      MODE == kNV;
    const bool mx32 = MODE != kNV && std::is_same<T, __nv_bfloat16>::value && vec && aligned32(x) && aligned32(y) &&
                      (mask == nullptr || aligned16(mask));
    if constexpr (MODE != kNV) {
      if (mx32) {
        const int64_t n32 = n / 32;
        auto run = [&](auto kernel) {
          launch_pdl(kernel, dim3((unsigned)persistent_grid(n32 + 1, (const void*)kernel, kThreads, QATF_MX32_CTAS)),
                     dim3(kThreads), stream, reinterpret_cast<const __nv_bfloat16*>(x),
                     reinterpret_cast<__nv_bfloat16*>(y), reinterpret_cast<uint32_t*>(mask), n32);
          return launch_status();
        };
        return mask != nullptr ? run(fp4_qdq_mx32_kernel<MODE, true>) : run(fp4_qdq_mx32_kernel<MODE, false>);
      }
    }
    if (wide) {
      const int64_t n16 = n / 16;
      auto run = [&](auto k) {
        launch_pdl(k, dim3((unsigned)persistent_grid(n16, (const void*)k, kThreads, QATF_NVW_CTAS)), dim3(kThreads),
                   stream, reinterpret_cast<const __nv_bfloat16*>(x), reinterpret_cast<__nv_bfloat16*>(y), mask, n16,
                   tensor_amax);
      };
      if (mask != nullptr) {
        run(fp4_qdq_bf16w_kernel<MODE, true>);
      } else {
        run(fp4_qdq_bf16w_kernel<MODE, false>);
      }
    } else if (vec) {
      const int64_t n_vec = n / VecTraits<T>::kVec;
      if (mask != nullptr) {
        auto k = fp4_qdq_vec_kernel<T, MODE, true>;
        fp4_qdq_vec_kernel<T, MODE, true><<<grid_for(n_vec / kUnroll + 1, (const void*)k), kThreads, 0, stream>>>(
            xt, yt, mask, n_vec, tensor_amax);
      } else {
        auto k = fp4_qdq_vec_kernel<T, MODE, false>;
        fp4_qdq_vec_kernel<T, MODE, false><<<grid_for(n_vec / kUnroll + 1, (const void*)k), kThreads, 0, stream>>>(
            xt, yt, mask, n_vec, tensor_amax);
      }
    } else {
      const int64_t groups = (n + 7) / 8;
      if (mask != nullptr) {
        auto k = fp4_qdq_generic_kernel<T, MODE, true>;
        fp4_qdq_generic_kernel<T, MODE, true><<<grid_for(groups, (const void*)k), kThreads, 0, stream>>>(
            xt, rows, cols, ld, yt, mask, tensor_amax);
      } else {
        auto k = fp4_qdq_generic_kernel<T, MODE, false>;
        fp4_qdq_generic_kernel<T, MODE, false><<<grid_for(groups, (const void*)k), kThreads, 0, stream>>>(
            xt, rows, cols, ld, yt, mask, tensor_amax);
      }
    }
    return launch_status();
  });
}

template <int MODE>
int fp4_pack(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float* tensor_amax,
             uint8_t* packed, uint8_t* scales, float* scale_2, void* recon, cudaStream_t stream) {
  constexpr int B = Fp4Consts<MODE>::kBlock;
  if (rows < 0 || cols < 0 || cols % B != 0 || ld < cols) return QATF_ERR_INVALID;
  if (rows > 0 && cols > 0 && (x == nullptr || packed == nullptr || scales == nullptr)) return QATF_ERR_INVALID;
  if (MODE == kNV && (tensor_amax == nullptr || scale_2 == nullptr)) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) {
    if (MODE == kNV) {
      // no block reads tensor_amax: still publish scale_2 like the reference
      return QATF_OK;
    }
    return QATF_OK;
  }
  return dispatch_dtype(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    const T* xt = static_cast<const T*>(x);
    T* rt = static_cast<T*>(recon);
    const int64_t n = rows * cols;
    const bool vec = (ld == cols) && aligned16(x) && (recon == nullptr || aligned16(recon)) &&
                     (reinterpret_cast<uintptr_t>(packed) % 4 == 0);
    const bool wide = std::is_same<T, __nv_bfloat16>::value && vec && aligned32(x) &&
                      (recon == nullptr || aligned32(recon)) && (reinterpret_cast<uintptr_t>(packed) % 8 == 0);
    if (wide) {
      const int64_t n16 = n / 16;
      auto k = fp4_pack_bf16w_kernel<MODE>;
      launch_pdl(k, dim3((unsigned)grid_for(n16, (const void*)k)), dim3(kThreads), stream,
                 reinterpret_cast<const __nv_bfloat16*>(x), n16, tensor_amax, packed, scales, scale_2,
                 reinterpret_cast<__nv_bfloat16*>(recon));
    } else if (vec) {
      const int64_t n_vec = n / VecTraits<T>::kVec;
      auto k = fp4_pack_vec_kernel<T, MODE>;
      fp4_pack_vec_kernel<T, MODE><<<grid_for(n_vec / kUnroll + 1, (const void*)k), kThreads, 0, stream>>>(
          xt, n_vec, tensor_amax, packed, scales, scale_2, rt);
    } else {
      auto k = fp4_pack_generic_kernel<T, MODE>;
      fp4_pack_generic_kernel<T, MODE><<<grid_for(n / 2, (const void*)k), kThreads, 0, stream>>>(
          xt, rows, cols, ld, tensor_amax, packed, scales, scale_2, rt);
    }
    return launch_status();
  });
}

}  // namespace qatf

using namespace qatf;

extern "C" {

int qatf_tensor_amax(const void* x, int dtype, int64_t n, float* amax_out, void* stream) {
  if (n < 0 || amax_out == nullptr || (n > 0 && x == nullptr)) return QATF_ERR_INVALID;
  launch_pdl(amax_zero_kernel, dim3(1), dim3(32), static_cast<cudaStream_t>(stream),
             reinterpret_cast<uint32_t*>(amax_out), (int64_t)1);
  const int st = launch_status();
  return st != QATF_OK ? st : qatf_tensor_amax_update(x, dtype, n, amax_out, stream);
}

int qatf_tensor_amax_update(const void* x, int dtype, int64_t n, float* amax_inout, void* stream) {
  if (n < 0 || amax_inout == nullptr || (n > 0 && x == nullptr)) return QATF_ERR_INVALID;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* amax_out = amax_inout;
  if (n == 0) return QATF_OK;
  return dispatch_dtype(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    const int vec_ok = aligned32(x) ? 1 : 0;
    const int64_t chunks = n / (32 / (int64_t)sizeof(T));
    auto k = amax_kernel<T, 2>;
    const int64_t grid = persistent_grid((chunks + 1) / 2, (const void*)k, kAmaxThreads);
    launch_pdl(k, dim3((unsigned)grid), dim3(kAmaxThreads), s, static_cast<const T*>(x), n, vec_ok,
               reinterpret_cast<uint32_t*>(amax_out));
    return launch_status();
  });
}

int qatf_tensor_amax_batched(const void* x, int dtype, int64_t batches, int64_t n, float* amax_out, void* stream) {
  if (batches < 0 || n < 0 || (batches > 0 && amax_out == nullptr) || (batches > 0 && n > 0 && x == nullptr))
    return QATF_ERR_INVALID;
  if (batches > 65535) return QATF_ERR_UNSUPPORTED;
  if (batches == 0) return QATF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  launch_pdl(amax_zero_kernel, dim3((unsigned)((batches + 127) / 128)), dim3(128), s,
             reinterpret_cast<uint32_t*>(amax_out), batches);
  if (const int st = launch_status(); st != QATF_OK || n == 0) return st;
  return dispatch_dtype(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    // every slice start is 32-byte aligned when the base is and a slice is a whole number of
    // 32-byte chunks
    const int vec_ok = (aligned32(x) && (n * (int64_t)sizeof(T)) % 32 == 0) ? 1 : 0;
    const int64_t chunks = n / (32 / (int64_t)sizeof(T));
    auto k = amax_kernel<T, 4>;
    const int64_t full = persistent_grid(INT64_MAX / 2, (const void*)k, kAmaxThreads);
    const int64_t per = std::max<int64_t>(
        1, std::min<int64_t>((full + batches - 1) / batches, (chunks + 4 * kAmaxThreads - 1) / (4 * kAmaxThreads)));
    launch_pdl(k, dim3((unsigned)per, (unsigned)batches), dim3(kAmaxThreads), s,
               static_cast<const T*>(x), n, vec_ok, reinterpret_cast<uint32_t*>(amax_out));
    return launch_status();
  });
}

int qatf_nvfp4_qdq(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float* tensor_amax, void* y,
                   uint8_t* mask_bits, void* stream) {
  return fp4_qdq<kNV>(x, dtype, rows, cols, ld, tensor_amax, y, mask_bits, static_cast<cudaStream_t>(stream));
}

int qatf_nvfp4_qdq_shadow(const float* latent, int64_t rows, int64_t cols, const float* tensor_amax, float* out,
                          uint8_t* mask_bits, void* stream) {
  if (rows < 0 || cols < 0 || cols % 16 != 0 || tensor_amax == nullptr) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (latent == nullptr || out == nullptr || mask_bits == nullptr) return QATF_ERR_INVALID;
  if (!aligned32(latent) || !aligned32(out) || (reinterpret_cast<uintptr_t>(mask_bits) & 1u) != 0)
    return QATF_ERR_INVALID;
  const int64_t n16 = rows * (cols / 16);
  auto k = nvfp4_qdq_shadow_kernel;  // one shard after another: programmatic dependent launch
  launch_pdl(k, dim3((unsigned)persistent_grid(n16, (const void*)k, kThreads, 3)), dim3(kThreads),
             static_cast<cudaStream_t>(stream), latent, out, mask_bits, n16, tensor_amax);
  return launch_status();
}

int qatf_nvfp4_fake_quant(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, float* amax_scratch,
                          void* y, uint8_t* mask_bits, void* stream) {
  if (amax_scratch == nullptr || rows < 0 || cols < 0 || ld < cols) return QATF_ERR_INVALID;
  if (rows > 0 && cols > 0 && ld != cols) return QATF_ERR_UNSUPPORTED;  // the amax pass reads a dense tensor
  int st = qatf_tensor_amax(x, dtype, rows * cols, amax_scratch, stream);
  if (st != QATF_OK) return st;
  return qatf_nvfp4_qdq(x, dtype, rows, cols, ld, amax_scratch, y, mask_bits, stream);
}

int qatf_nvfp4_pack(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, const float* tensor_amax,
                    uint8_t* packed, uint8_t* scales, float* weight_scale_2, void* recon, void* stream) {
  return fp4_pack<kNV>(x, dtype, rows, cols, ld, tensor_amax, packed, scales, weight_scale_2, recon,
                       static_cast<cudaStream_t>(stream));
}

int qatf_nvfp4_dequant(const uint8_t* packed, const uint8_t* scales, const float* weight_scale_2, int64_t rows,
                       int64_t cols, float* out, void* stream) {
  if (rows < 0 || cols < 0 || cols % 16 != 0) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (packed == nullptr || scales == nullptr || weight_scale_2 == nullptr || out == nullptr) return QATF_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(packed) & 1u) == 0 && aligned16(out)) {
    auto k = fp4_dequant_vec_kernel<kNV>;
    const int64_t n4 = rows * cols / 4;
    k<<<grid_for(n4 / 4 + 1, (const void*)k), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint16_t*>(packed), scales, weight_scale_2, n4, reinterpret_cast<float4*>(out));
    return launch_status();
  }
  auto k = nvfp4_dequant_kernel;
  nvfp4_dequant_kernel<<<grid_for(rows * cols / 2, (const void*)k), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, scales, weight_scale_2, rows, cols, out);
  return launch_status();
}

int qatf_mxfp4_qdq_even(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, void* y, uint8_t* mask_bits,
                        void* stream) {
  return fp4_qdq<kMXEven>(x, dtype, rows, cols, ld, nullptr, y, mask_bits, static_cast<cudaStream_t>(stream));
}

int qatf_mxfp4_qdq_ceil(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, void* y, void* stream) {
  return fp4_qdq<kMXCeil>(x, dtype, rows, cols, ld, nullptr, y, nullptr, static_cast<cudaStream_t>(stream));
}

int qatf_mxfp4_pack(const void* x, int dtype, int64_t rows, int64_t cols, int64_t ld, uint8_t* packed, uint8_t* scales,
                    void* recon, void* stream) {
  return fp4_pack<kMXEven>(x, dtype, rows, cols, ld, nullptr, packed, scales, nullptr, recon,
                           static_cast<cudaStream_t>(stream));
}

int qatf_mxfp4_dequant(const uint8_t* packed, const uint8_t* scales, int64_t rows, int64_t cols, float* out,
                       void* stream) {
  if (rows < 0 || cols < 0 || cols % 32 != 0) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (packed == nullptr || scales == nullptr || out == nullptr) return QATF_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(packed) & 1u) == 0 && aligned16(out)) {
    auto k = fp4_dequant_vec_kernel<kMXEven>;
    const int64_t n4 = rows * cols / 4;
    k<<<grid_for(n4 / 4 + 1, (const void*)k), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        reinterpret_cast<const uint16_t*>(packed), scales, nullptr, n4, reinterpret_cast<float4*>(out));
    return launch_status();
  }
  auto k = mxfp4_dequant_kernel;
  mxfp4_dequant_kernel<<<grid_for(rows * cols / 2, (const void*)k), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      packed, scales, rows, cols, out);
  return launch_status();
}

int qatf_ste_backward(const void* grad_out, int dtype, int64_t n, const uint8_t* mask_bits, void* grad_in,
                      void* stream) {
  if (n < 0 || (n > 0 && (grad_out == nullptr || mask_bits == nullptr || grad_in == nullptr))) return QATF_ERR_INVALID;
  if (n == 0) return QATF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  return dispatch_dtype(dtype, [&](auto tag) -> int {
    using T = decltype(tag);
    constexpr int VEC = VecTraits<T>::kVec;
    if (std::is_same<T, __nv_bfloat16>::value && n % 16 == 0 && aligned32(grad_out) && aligned32(grad_in) &&
        (reinterpret_cast<uintptr_t>(mask_bits) & 1u) == 0) {
      auto k = ste_bf16w_kernel;
      launch_pdl(k, dim3((unsigned)grid_for(n / 16, (const void*)k)), dim3(kThreads), s,
                 static_cast<const __nv_bfloat16*>(grad_out), reinterpret_cast<const uint16_t*>(mask_bits),
                 static_cast<__nv_bfloat16*>(grad_in), n / 16);
    } else if (n % VEC == 0 && aligned16(grad_out) && aligned16(grad_in)) {
      auto k = ste_vec_kernel<T>;
      ste_vec_kernel<T><<<grid_for(n / VEC, (const void*)k), kThreads, 0, s>>>(
          static_cast<const T*>(grad_out), mask_bits, static_cast<T*>(grad_in), n / VEC);
    } else {
      auto k = ste_generic_kernel<T>;
      ste_generic_kernel<T><<<grid_for(n, (const void*)k), kThreads, 0, s>>>(static_cast<const T*>(grad_out),
                                                                           mask_bits, static_cast<T*>(grad_in), n);
    }
    return launch_status();
  });
}

int qatf_e2m1_pack_rows(const uint8_t* nibbles, int64_t rows, int64_t cols, uint8_t* packed, void* stream) {
  if (rows < 0 || cols < 0 || cols % 2 != 0) return QATF_ERR_INVALID;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (nibbles == nullptr || packed == nullptr) return QATF_ERR_INVALID;
  auto k = e2m1_pack_rows_kernel;
  e2m1_pack_rows_kernel<<<grid_for(rows * cols / 2, (const void*)k), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      nibbles, rows * cols / 2, packed);
  return launch_status();
}

int qatf_e2m1_unpack_rows(const uint8_t* packed, int64_t rows, int64_t packed_cols, uint8_t* nibbles, void* stream) {
  if (rows < 0 || packed_cols < 0) return QATF_ERR_INVALID;
  if (rows == 0 || packed_cols == 0) return QATF_OK;
  if (nibbles == nullptr || packed == nullptr) return QATF_ERR_INVALID;
  auto k = e2m1_unpack_rows_kernel;
  e2m1_unpack_rows_kernel<<<grid_for(rows * packed_cols, (const void*)k), kThreads, 0,
                            static_cast<cudaStream_t>(stream)>>>(packed, rows * packed_cols, nibbles);
  return launch_status();
}

int qatf_nvfp4_operand(const void* x, int dtype, int64_t rows, int64_t cols, const float* tensor_amax, int role,
                       uint8_t* codes, uint8_t* scales, void* deq, uint8_t* mask_bits, void* stream) {
  return qatf_nvfp4_operand_tracked(x, dtype, rows, cols, tensor_amax, role, codes, scales, deq, mask_bits, nullptr,
                                    stream);
}

int qatf_nvfp4_operand_tracked(const void* x, int dtype, int64_t rows, int64_t cols, const float* tensor_amax,
                               int role, uint8_t* codes, uint8_t* scales, void* deq, uint8_t* mask_bits,
                               float* running_amax, void* stream) {
  if (rows < 0 || cols < 0 || (role != QATF_OPERAND_A && role != QATF_OPERAND_B)) return QATF_ERR_INVALID;
  if (rows % (role == QATF_OPERAND_A ? 128 : 256) != 0 || cols % (role == QATF_OPERAND_A ? 128 : 64) != 0)
    return QATF_ERR_UNSUPPORTED;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (dtype != QATF_BF16) return QATF_ERR_DTYPE;
  if (x == nullptr || tensor_amax == nullptr || codes == nullptr || scales == nullptr) return QATF_ERR_INVALID;
  if (!aligned32(x) || (deq != nullptr && !aligned32(deq)) || !aligned16(codes) || !aligned16(scales) ||
      (mask_bits != nullptr && !aligned16(mask_bits)) || (reinterpret_cast<uintptr_t>(running_amax) & 3u) != 0)
    return QATF_ERR_INVALID;
  const int64_t n16 = rows * (cols / 16);
  if (n16 >= (int64_t(1) << 32)) return QATF_ERR_UNSUPPORTED;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* db = static_cast<__nv_bfloat16*>(deq);
  auto* rb = reinterpret_cast<uint32_t*>(running_amax);
  const uint32_t cols16 = (uint32_t)(cols / 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (role == QATF_OPERAND_A) {
    auto k = nvfp4_operand_bf16_kernel<QATF_OPERAND_A>;
    k<<<persistent_grid(n16, (const void*)k, kThreads, kOperandCtas<QATF_OPERAND_A>), kThreads, 0, s>>>(
        xb, n16, cols16, tensor_amax, codes, scales, db, mask_bits, rb);
  } else {
    auto k = nvfp4_operand_bf16_kernel<QATF_OPERAND_B>;
    k<<<persistent_grid(n16, (const void*)k, kThreads, kOperandCtas<QATF_OPERAND_B>), kThreads, 0, s>>>(
        xb, n16, cols16, tensor_amax, codes, scales, db, mask_bits, rb);
  }
  return launch_status();
}

int qatf_mxfp4_operand(const void* x, int dtype, int64_t rows, int64_t cols, int role, int rule, uint8_t* codes,
                       uint8_t* scales, void* deq, uint8_t* mask_bits, void* stream) {
  if (rows < 0 || cols < 0 || (role != QATF_OPERAND_A && role != QATF_OPERAND_B) ||
      (rule != QATF_MXFP4_EVEN && rule != QATF_MXFP4_CEIL))
    return QATF_ERR_INVALID;
  if (rows % (role == QATF_OPERAND_A ? 128 : 256) != 0 || cols % (role == QATF_OPERAND_A ? 256 : 128) != 0)
    return QATF_ERR_UNSUPPORTED;
  if (rows == 0 || cols == 0) return QATF_OK;
  if (dtype != QATF_BF16) return QATF_ERR_DTYPE;
  if (x == nullptr || codes == nullptr || scales == nullptr) return QATF_ERR_INVALID;
  if (!aligned32(x) || (deq != nullptr && !aligned32(deq)) || !aligned16(codes) || !aligned16(scales) ||
      (mask_bits != nullptr && !aligned16(mask_bits)))
    return QATF_ERR_INVALID;
  const int64_t n16 = rows * (cols / 16);
  if (n16 >= (int64_t(1) << 32)) return QATF_ERR_UNSUPPORTED;
  const auto* xb = static_cast<const __nv_bfloat16*>(x);
  auto* db = static_cast<__nv_bfloat16*>(deq);
  const uint32_t cols16 = (uint32_t)(cols / 16);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  auto run = [&](auto kernel) {
    launch_pdl(kernel, dim3((unsigned)persistent_grid(n16, (const void*)kernel, kThreads, 3)), dim3(kThreads), s, xb,
               n16, cols16, codes, scales, db, mask_bits);
  };
  if (role == QATF_OPERAND_A) {
    if (rule == QATF_MXFP4_EVEN) run(mxfp4_operand_bf16_kernel<QATF_OPERAND_A, kMXEven>);
    else run(mxfp4_operand_bf16_kernel<QATF_OPERAND_A, kMXCeil>);
  } else {
    if (rule == QATF_MXFP4_EVEN) run(mxfp4_operand_bf16_kernel<QATF_OPERAND_B, kMXEven>);
    else run(mxfp4_operand_bf16_kernel<QATF_OPERAND_B, kMXCeil>);
  }
  return launch_status();
}

int qatf_nvfp4_qdq_experts(const void* x, int dtype, int64_t experts, int64_t rows, int64_t cols,
                           const float* tensor_amax, void* y, uint8_t* mask_bits, void* stream) {
  if (experts < 0 || rows < 0 || cols < 0 || cols % 16 != 0) return QATF_ERR_INVALID;
  if (experts == 0 || rows == 0 || cols == 0) return QATF_OK;
  if (x == nullptr || y == nullptr || tensor_amax == nullptr) return QATF_ERR_INVALID;
  if (experts > 65535) return QATF_ERR_UNSUPPORTED;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t per = rows * cols;
  if (dtype == QATF_BF16 && aligned32(x) && aligned32(y)) {
    // one launch: the x grid covers an expert, the y grid the experts
    const int64_t n16 = per / 16;
    auto run = [&](auto kernel) {
      const int64_t full = grid_for(experts * n16, (const void*)kernel);
      const int64_t gx = std::max<int64_t>(1, std::min<int64_t>((n16 + kThreads - 1) / kThreads,
                                                                (full + experts - 1) / experts));
      kernel<<<dim3((unsigned)gx, (unsigned)experts), kThreads, 0, s>>>(
          static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), mask_bits, n16, tensor_amax);
      return launch_status();
    };
    return mask_bits != nullptr ? run(fp4_qdq_bf16w_kernel<kNV, true>) : run(fp4_qdq_bf16w_kernel<kNV, false>);
  }
  // other dtypes and alignments: expert by expert through the 2-D entry point
  const int64_t esz = dtype == QATF_F32 ? 4 : 2;
  for (int64_t e = 0; e < experts; ++e) {
    const int st = fp4_qdq<kNV>(static_cast<const uint8_t*>(x) + e * per * esz, dtype, rows, cols, cols,
                                tensor_amax + e, static_cast<uint8_t*>(y) + e * per * esz,
                                mask_bits != nullptr ? mask_bits + e * per / 8 : nullptr, s);
    if (st != QATF_OK) return st;
  }
  return QATF_OK;
}

}  // extern "C"
