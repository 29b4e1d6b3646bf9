// tcgen05 GEMMs of the NVFP4 and MXFP4 W4A4 quantized linears (sm_100a).
//
//   forward   Y  = X_q W_q^T           block-scaled FP4 x FP4 (kind::mxf4nvf4 with UE4M3 block-16
//                                      scales, or kind::mxf4 with UE8M0 block-32 scales for
//                                      MXFP4Linear, mxfp4.py:285-290), FP32 accumulators in
//                                      TMEM, BF16 out
//   backward  dX = (dY W_q) * mask_x    BF16 x BF16 (kind::f16), STE mask applied in the epilogue
//             dW = (dY^T X_q) * mask_w  BF16 x BF16 with both operands MN-major
//
// Semantics: NVFP4Linear.forward with _quantize_activations (qatfactory/quant/formats/nvfp4.py:
// 636-658) is F.linear(fq(X), fq(W)); autograd then gives dX = STE_x(dY @ W_q) and
// dW = STE_w(dY^T @ X_q) (nvfp4.py:32-41).  The FP4 GEMM multiplies the E2M1 codes and E4M3
// block scales exactly and applies the two FP32 tensor scales (amax / 2688) in the epilogue.
//
// A persistent CTA per SM walks 128 x 256 output tiles with warp-specialised roles:
//   warp 0      TMA producer (one lane): A/B tiles (128-byte swizzle) and, for FP4, the scale
//               factor atoms (1-D bulk copies) into a 4-stage shared-memory ring
//   warp 1      allocates TMEM; one lane issues tcgen05.cp (scales) and tcgen05.mma, and
//               tcgen05.commit frees each stage and signals each finished accumulator
//   warps 2..   epilogue (4 warps for BF16 with two TMEM accumulators, 8 for FP4 with one):
//               tcgen05.ld 32 lanes x 32 columns at a time, scale / mask, 32-byte BF16 stores
// Every mbarrier wait is bounded (2 s of %globaltimer); a wait that expires sets
// the caller's error word and a CTA-wide abort flag, every role leaves its loop, and TMEM is
// freed before the CTA exits.  CTAs that start after an error return at once.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "qatf.h"
#include "qatf_common.cuh"
#include "qatf_fp4.cuh"
#include "qatf_tma.cuh"

namespace qatf {
namespace tc {

constexpr int kBM = 128;
constexpr int kBN = 256;
constexpr int kRowBytes = 128;           // one 128-byte swizzle row per operand row and stage
constexpr int kTileA = kBM * kRowBytes;  // 16 KB
constexpr int kTileB = kBN * kRowBytes;  // 32 KB
constexpr uint64_t kTimeoutNs = 2000000000ull;

enum Kind : int { kKindBF16 = 0, kNVF4 = 1, kMXF4 = 2 };
__host__ __device__ constexpr bool is_fp4(int kind) { return kind == kNVF4 || kind == kMXF4; }

// Shared memory of the single-CTA kernel.  Per 256-column K stage, NVFP4 also carries the A
// scale blocks (2 x 4 KB: 128 rows x 2 K-blocks of 64 each) and the B scale blocks (4 x 4 KB:
// 256 rows x 1 K-block each), one 128x256b TMEM copy per block; MXFP4, whose block-32 scale
// word spans 128 columns, half as many (A 1 x 4 KB: 128 rows x 2 K-blocks of 128; B 2 x 4 KB:
// 256 rows x 1 K-block of 128).  FP4 keeps three stages where BF16 keeps four.
template <int KIND>
struct SmemLayout {
  static constexpr int stages = is_fp4(KIND) ? 3 : 4;
  static constexpr int sfa_bytes = KIND == kNVF4 ? 2 * 4096 : (KIND == kMXF4 ? 4096 : 0);
  static constexpr int sfb_bytes = KIND == kNVF4 ? 4 * 4096 : (KIND == kMXF4 ? 2 * 4096 : 0);
  static constexpr int a = 0;
  static constexpr int b = a + stages * kTileA;
  static constexpr int sfa = b + stages * kTileB;
  static constexpr int sfb = sfa + stages * sfa_bytes;
  static constexpr int bars = sfb + stages * sfb_bytes;  // full[S], empty[S], acc_full[2], acc_empty[2]
  static constexpr int holder = bars + (2 * stages + 4) * 8;
  static constexpr int flags = holder + 8;
  static constexpr int end = flags + 8;
  static constexpr int bytes = end + 1024;  // slack to align the base to 1024 bytes
};

// ------------------------------------------------------------------------ PTX wrappers
// Bounded wait for the phase with the given parity.  Returns false if the CTA is aborting or
// the wait ran past the limit (then the abort flag and the error word are set).  The first
// try is inline; only a wait that has to spin leaves the caller's instruction stream.
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 31u) == 0u) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicOr(err, 1);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag, int* err) {
  return mbar_try_wait(bar, parity) || mbar_wait_slow(bar, parity, abort_flag, err);
}

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait until a readiness counter that other CTAs' quantizer warps release reaches
// `target` (acquire, GPU scope).  Same limit and error handling as mbar_wait (error bit 2).
__device__ __noinline__ bool ready_wait_slow(const uint32_t* flag, uint32_t target, volatile int* abort_flag,
                                             int* err) {
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (ld_acquire_gpu(flag) >= target) return true;
    __nanosleep(32);
    if ((i & 15u) == 0u) {
      if (*abort_flag) return false;
      if (global_ns() - t0 > kTimeoutNs) {
        *abort_flag = 1;
        atomicOr(err, 2);
        return false;
      }
    }
  }
}

__device__ __forceinline__ bool ready_wait(const uint32_t* flag, uint32_t target, volatile int* abort_flag, int* err) {
  return ld_acquire_gpu(flag) >= target || ready_wait_slow(flag, target, abort_flag, err);
}

__device__ __forceinline__ void bulk_load(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}

__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_nvf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                         uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

__device__ __forceinline__ void mma_mxf4(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                         uint32_t sfb, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
      : "memory");
}

// 128 rows x 32 bytes of shared memory (core matrices of 8 rows x 16 bytes: halves 128 bytes
// apart, 8-row groups 256 bytes apart) into 8 TMEM columns of all 128 lanes.
__device__ __forceinline__ void sf_copy_wide(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor (tcgen05 format, version 1): start, leading and stride byte
// offsets in 16-byte units; layout 2 = 128-byte swizzle, 0 = no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)((lbo >> 4) & 0x3FFFu) << 16) |
         ((uint64_t)((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46) | ((uint64_t)layout << 61);
}

// Instruction descriptors, M = 128, N = 256.
//   kind::f16:     D F32 (bits 4-5 = 1), A/B BF16 (bits 7-9, 10-12 = 1), majors (bits 15, 16)
//   kind::mxf4nvf4: A/B E2M1 (= 1), UE4M3 scales (bit 23 = 0), scale ids 0, K = 64
constexpr uint32_t kIdescShape = ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
__host__ __device__ constexpr uint32_t idesc_bf16(bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | kIdescShape;
}
constexpr uint32_t kIdescNvf4 = (1u << 7) | (1u << 10) | kIdescShape;
//   kind::mxf4:     A/B E2M1 (= 1), UE8M0 scales (bit 23 = 1), K = 64; the scale-factor ids
//                   (A bits 29-30, B bits 4-5) pick the first byte of each 32-bit scale word the
//                   MMA reads (its two block-32 scales), 0 or 2
__host__ __device__ constexpr uint32_t idesc_mxf4(uint32_t sf_id) {
  return (1u << 7) | (1u << 10) | (1u << 23) | (sf_id << 29) | (sf_id << 4) | kIdescShape;
}

struct Args {
  int m_tiles, n_tiles, k_tiles;
  const uint8_t* sfa;
  const uint8_t* sfb;
  const float* a_amax;
  const float* b_amax;
  __nv_bfloat16* out;
  int64_t ldo;
  const uint8_t* mask;  // STE bits over out's flat index, or null
  int* err;
  // activation quantization inside the kernel (qatf_nvfp4_linear_fwd): X BF16 [M, K] with the
  // tensor amax a_amax; the quantizer warps write X's codes (read back through map_a), its
  // A-side scale blocks (sfa), deq and mask, and count finished 32-row quarter panels in
  // ready[mt * k_tiles + kt]
  const __nv_bfloat16* x;
  uint8_t* xq_codes;
  uint8_t* xq_sf;
  __nv_bfloat16* xq_deq;
  uint8_t* xq_mask;
  uint32_t* ready;
  uint32_t* work;  // next quantization item (zero at launch)
  // split-K of the last partial wave (CTA-pair BF16 kernel): tiles >= full_units are done as
  // `split` K-slices each, whose FP32 partial tiles go to ws[unit][256][256] and are summed by
  // splitk_reduce_kernel; split == 0: every tile whole
  int split;
  int full_units;
  float* ws;
};

// Tile t of the persistent schedule: groups of kGroupM row tiles, column tiles outer inside a
// group, so the CTAs of one wave share a few A row panels and walk B together (L2 reuse).
constexpr int kGroupM = 8;
__device__ __forceinline__ void tile_coords(int t, int m_tiles, int n_tiles, int& mt, int& nt) {
  const int per_group = kGroupM * n_tiles;
  const int g = t / per_group;
  const int r = t - g * per_group;
  const int gm = min(kGroupM, m_tiles - g * kGroupM);
  mt = g * kGroupM + r % gm;
  nt = r / gm;
}

// Work unit u of the CTA-pair schedule: a whole 256 x 256 tile (part < 0), or K-slice
// u - full_units of a tail tile (K tiles [k0, k1), partial tile `part` of the workspace).
struct PairUnit {
  int mp, nt, k0, k1, part;
};
__device__ __forceinline__ PairUnit pair_unit(int u, int m_pairs, const Args& a) {
  PairUnit r;
  if (a.split <= 0 || u < a.full_units) {
    tile_coords(u, m_pairs, a.n_tiles, r.mp, r.nt);
    r.k0 = 0;
    r.k1 = a.k_tiles;
    r.part = -1;
  } else {
    const int v = u - a.full_units;
    const int sl = v % a.split;
    tile_coords(a.full_units + v / a.split, m_pairs, a.n_tiles, r.mp, r.nt);
    r.k0 = (int)((int64_t)a.k_tiles * sl / a.split);
    r.k1 = (int)((int64_t)a.k_tiles * (sl + 1) / a.split);
    r.part = v;
  }
  return r;
}

// ----------------------------------------------------------------------------- kernel
// Persistent: one CTA per SM walks tiles blockIdx.x, +gridDim.x, ...  The shared-memory ring,
// its phases and the accumulator buffers carry over from tile to tile, so loads for the next
// tile stream in while the epilogue drains the previous one.
//   NACC = 2: two TMEM accumulators (512 columns); the MMA warp fills one while the epilogue
//             drains the other.
//   NACC = 1: one accumulator (FP4: its scale factors take the remaining columns); EPI epilogue
//             warps (8) pull the whole tile into registers, release TMEM, then convert and store.
//   FUSE_A:   ten more warps quantize the BF16 activation X into the A operand while the GEMM
//             runs (qatf_nvfp4_linear_fwd): work items of 32 rows x 256 K, taken from a global
//             counter by every CTA's quantizer warps in the order the tile schedule consumes
//             them; the producer waits for an A stage's four quarter panels before loading it.
//             20 warps (at most 96 registers a thread): 0 producer, 1 MMA, 4..11 epilogue
//             (warp % 4 is the TMEM lane quarter each reads), 2, 3 and 12..19 quantizers.
constexpr int kFusedThreads = 640;
template <int KIND, bool A_MN, bool B_MN, int NACC, int EPI, bool FUSE_A = false>
__global__ void __launch_bounds__(FUSE_A ? kFusedThreads : 64 + 32 * EPI, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                   const Args args) {
  using L = SmemLayout<KIND>;
  constexpr int kStages = L::stages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  const uint32_t bar_full = s0 + L::bars;
  const uint32_t bar_empty = bar_full + kStages * 8;
  const uint32_t bar_acc_full = bar_empty + kStages * 8;
  const uint32_t bar_acc_empty = bar_acc_full + 2 * 8;
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + L::holder);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::flags);
  constexpr uint32_t kTmemCols = 512u;
  constexpr uint32_t kSfaCol = NACC * kBN;   // 16 columns: 4 K-blocks x 4
  constexpr uint32_t kSfbCol = kSfaCol + 16;  // 32 columns: 4 K-blocks x 8
  static_assert(!is_fp4(KIND) || NACC * kBN + 48 <= 512, "TMEM columns");
  static_assert(EPI == 4 || EPI == 8, "epilogue warps");
  constexpr int kColsPerWarp = kBN * 4 / EPI;  // 256 (4 warps) or 128 (8 warps)
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_total = args.m_tiles * args.n_tiles;
  constexpr int kEpiFirst = FUSE_A ? 4 : 2;  // first epilogue warp
  static_assert(!FUSE_A || (KIND == kNVF4 && EPI == 8), "the fused kernel is the FP4 kernel");

  // an earlier CTA gave up: leave before any collective tcgen05 operation (CTA-uniform)
  if (threadIdx.x == 0) *abort_flag = *reinterpret_cast<volatile int*>(args.err);
  __syncthreads();
  if (*abort_flag != 0) return;
  __syncthreads();

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_acc_full + 8 * b, 1);
      mbar_init(bar_acc_empty + 8 * b, EPI);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tmem = *holder;
  const int kt_n = args.k_tiles;

  auto role_producer = [&]() {
    // ------------------------------------------------------------------- producer
    constexpr uint32_t tx = kTileA + kTileB + (is_fp4(KIND) ? L::sfa_bytes + L::sfb_bytes : 0);
    uint32_t it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_total && ok; t += gridDim.x) {
      int mt, nt;
      tile_coords(t, args.m_tiles, args.n_tiles, mt, nt);
      const int m0 = mt * kBM, n0 = nt * kBN;
      for (int kt = 0; kt < kt_n; ++kt, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(bar_empty + 8 * s, ((it / kStages) & 1) ^ 1, abort_flag, args.err)) {
          ok = false;
          break;
        }
        if constexpr (FUSE_A) {
          // the stage's sixteen panels are quantized; their writers fenced the stores to
          // the async proxy before the release, and this fence orders the TMA reads after it
          if (!ready_wait(args.ready + (int64_t)mt * kt_n + kt, 16u, abort_flag, args.err)) {
            ok = false;
            break;
          }
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        const uint32_t full = bar_full + 8 * s;
        mbar_expect_tx(full, tx);
        const uint32_t sa = s0 + L::a + s * kTileA;
        const uint32_t sb = s0 + L::b + s * kTileB;
        // K coordinate of this stage: 128 bytes = 64 BF16 or 256 FP4 (x in tensor-map elements)
        const int kx = is_fp4(KIND) ? kt * 128 : kt * 64;
        if (A_MN) {
          for (int c = 0; c < kBM / 64; ++c) tma_load_2d(sa + c * 64 * kRowBytes, &map_a, full, m0 + 64 * c, kt * 64);
        } else {
          tma_load_2d(sa, &map_a, full, kx, m0);
        }
        if (B_MN) {
          for (int c = 0; c < kBN / 64; ++c) tma_load_2d(sb + c * 64 * kRowBytes, &map_b, full, n0 + 64 * c, kt * 64);
        } else {
          tma_load_2d(sb, &map_b, full, kx, n0);
        }
        if constexpr (is_fp4(KIND)) {
          const uint32_t ssa = s0 + L::sfa + s * L::sfa_bytes;
          const uint32_t ssb = s0 + L::sfb + s * L::sfb_bytes;
          bulk_load(ssa, args.sfa + ((int64_t)mt * kt_n + kt) * L::sfa_bytes, L::sfa_bytes, full);
          bulk_load(ssb, args.sfb + ((int64_t)nt * kt_n + kt) * L::sfb_bytes, L::sfb_bytes, full);
        }
      }
    }
  };
  auto role_mma = [&]() {
    // ------------------------------------------------------------------ MMA issuer
    // stage-0 descriptors; a stage or K step moves only the start-address field (16-byte
    // units): 16 BF16 / 64 FP4 of K are 32 bytes along a K-major row, or 16 rows (2 KB) of an
    // MN-major tile
    const uint64_t desc_a0 = A_MN ? smem_desc(s0 + L::a, 64 * kRowBytes, 1024, 2) : smem_desc(s0 + L::a, 16, 1024, 2);
    const uint64_t desc_b0 = B_MN ? smem_desc(s0 + L::b, 64 * kRowBytes, 1024, 2) : smem_desc(s0 + L::b, 16, 1024, 2);
    constexpr uint64_t kStepA = A_MN ? 2048 / 16 : 32 / 16;
    constexpr uint64_t kStepB = B_MN ? 2048 / 16 : 32 / 16;
    uint32_t it = 0;
    int li = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < n_total && ok; t += gridDim.x, ++li) {
      const int b = li % NACC;
      if (!mbar_wait(bar_acc_empty + 8 * b, ((li / NACC) & 1) ^ 1, abort_flag, args.err)) break;
      fence_after();
      const uint32_t acc = tmem + b * kBN;
      for (int kt = 0; kt < kt_n; ++kt, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(bar_full + 8 * s, (it / kStages) & 1, abort_flag, args.err)) {
          ok = false;
          break;
        }
        fence_after();
        if constexpr (KIND == kNVF4) {
          const uint32_t ssa = s0 + L::sfa + s * L::sfa_bytes;
          const uint32_t ssb = s0 + L::sfb + s * L::sfb_bytes;
          // scale blocks into TMEM: A as 4 columns per K-block (column c of a lane holds row
          // 32c + lane%32), B as 8 columns per K-block (column h: row 32h + lane%32), both
          // replicated in all four lane quarters; the MMAs take 4-column-aligned addresses
#pragma unroll
          for (int h = 0; h < 2; ++h) sf_copy_wide(tmem + kSfaCol + 8 * h, smem_desc(ssa + 4096 * h, 128, 256, 0));
#pragma unroll
          for (int j = 0; j < 4; ++j) sf_copy_wide(tmem + kSfbCol + 8 * j, smem_desc(ssb + 4096 * j, 128, 256, 0));
          const uint64_t da = desc_a0 + (uint64_t)((s * kTileA) >> 4);
          const uint64_t db = desc_b0 + (uint64_t)((s * kTileB) >> 4);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_nvf4(acc, da + 2 * j, db + 2 * j, kIdescNvf4, tmem + kSfaCol + 4 * j, tmem + kSfbCol + 8 * j,
                     (kt | j) != 0);
        } else if constexpr (KIND == kMXF4) {
          const uint32_t ssa = s0 + L::sfa + s * L::sfa_bytes;
          const uint32_t ssb = s0 + L::sfb + s * L::sfb_bytes;
          // one A block (K-blocks of 128 at columns 0-3 and 4-7) and two B blocks (8 columns
          // each); the K = 64 MMA j reads bytes 2 (j % 2) and 2 (j % 2) + 1 of the words of
          // K-block j / 2, selected by the scale-factor ids of its instruction descriptor
          sf_copy_wide(tmem + kSfaCol, smem_desc(ssa, 128, 256, 0));
#pragma unroll
          for (int h = 0; h < 2; ++h) sf_copy_wide(tmem + kSfbCol + 8 * h, smem_desc(ssb + 4096 * h, 128, 256, 0));
          const uint64_t da = desc_a0 + (uint64_t)((s * kTileA) >> 4);
          const uint64_t db = desc_b0 + (uint64_t)((s * kTileB) >> 4);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_mxf4(acc, da + 2 * j, db + 2 * j, idesc_mxf4(2u * (j & 1)), tmem + kSfaCol + 4 * (j >> 1),
                     tmem + kSfbCol + 8 * (j >> 1), (kt | j) != 0);
        } else {
          const uint64_t da = desc_a0 + (uint64_t)((s * kTileA) >> 4);
          const uint64_t db = desc_b0 + (uint64_t)((s * kTileB) >> 4);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_bf16(acc, da + kStepA * j, db + kStepB * j, idesc_bf16(A_MN, B_MN), (kt | j) != 0);
        }
        mma_commit(bar_empty + 8 * s);
      }
      if (ok) mma_commit(bar_acc_full + 8 * b);
    }
  };
  auto role_epilogue = [&]() {
    // -------------------------------------------------------------------- epilogue
    const int e = warp - kEpiFirst;
    const int q = warp & 3;                       // TMEM lane quarter this warp may read
    const int c_base = (e / 4) * kColsPerWarp;    // column range of this warp
    float alpha = 1.0f;
    if constexpr (KIND == kNVF4) alpha = __fdiv_rn(args.a_amax[0], 2688.0f) * __fdiv_rn(args.b_amax[0], 2688.0f);
    int li = 0;
    for (int t = blockIdx.x; t < n_total; t += gridDim.x, ++li) {
      const int b = li % NACC;
      if (!mbar_wait(bar_acc_full + 8 * b, (li / NACC) & 1, abort_flag, args.err)) break;
      fence_after();
      int mt, nt;
      tile_coords(t, args.m_tiles, args.n_tiles, mt, nt);
      const int64_t row = (int64_t)mt * kBM + 32 * q + lane;
      const int64_t col0 = (int64_t)nt * kBN + c_base;
      __nv_bfloat16* orow = args.out + row * args.ldo + col0;
      const uint32_t tbase = tmem + b * kBN + ((uint32_t)(32 * q) << 16) + c_base;
      auto store_chunk = [&](const uint32_t (&r)[32], int c) {
        uint32_t keep = 0xFFFFFFFFu;
        if (args.mask != nullptr) keep = *reinterpret_cast<const uint32_t*>(args.mask + (row * args.ldo + col0 + 32 * c) / 8);
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float lo = __uint_as_float(r[2 * i]);
          float hi = __uint_as_float(r[2 * i + 1]);
          if constexpr (KIND == kNVF4) {
            lo *= alpha;
            hi *= alpha;
          }
          uint32_t v = pack_bf16x2(lo, hi);
          if (!((keep >> (2 * i)) & 1u)) v &= 0xFFFF0000u;
          if (!((keep >> (2 * i + 1)) & 1u)) v &= 0x0000FFFFu;
          o[i] = v;
        }
        st256(orow + 32 * c, o);
        st256(orow + 32 * c + 16, o + 8);
      };
      if constexpr (NACC == 1) {
        // pull the whole column range into registers as BF16 pairs (the output's bits, scaled
        // and rounded exactly as store_chunk does), hand the accumulator back, then store
        static_assert(is_fp4(KIND), "the one-accumulator epilogue has no STE mask");
        uint32_t o[kColsPerWarp / 32][16];
#pragma unroll
        for (int c = 0; c < kColsPerWarp / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + 32 * c, r);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            o[c][i] = pack_bf16x2(__uint_as_float(r[2 * i]) * alpha, __uint_as_float(r[2 * i + 1]) * alpha);
        }
        fence_before();
        __syncwarp();
        if (lane == 0) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar_acc_empty + 8 * b) : "memory");
#pragma unroll
        for (int c = 0; c < kColsPerWarp / 32; ++c) {
          st256(orow + 32 * c, o[c]);
          st256(orow + 32 * c + 16, o[c] + 8);
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < kColsPerWarp / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(tbase + 32 * c, r);
          if (c == kColsPerWarp / 32 - 1) {
            fence_before();
            __syncwarp();
            if (lane == 0)
              asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar_acc_empty + 8 * b) : "memory");
          }
          store_chunk(r, c);
        }
      }
    }
  };
  auto role_quantizer = [&]() {
    // ------------------------------------------------------------ activation quantizer
    // Item = (M tile mt, K stage kc, 32-row quarter, 64-column slice): 128 blocks, lane l
    // taking block 4 (l / 4) ... of rows mt*128 + quarter*32 + 8i + l/4 (i = 0..3) and 16-column
    // block 16 kc + 4 slice + l%4, so each group of four lanes reads one row's 128 contiguous
    // bytes and holds one 64-column K-block (one scale word).  Items run group by group of the
    // tile schedule (kGroupM M tiles), K stage outer: small items, so the stages the first
    // tiles need are done early instead of many stages being half done.
    const NvGlobal g = load_global<kNV>(args.a_amax);
    const uint32_t cols16 = (uint32_t)kt_n * 16u;
    const uint32_t atoms_k = cols16 >> 2;
    constexpr uint32_t kItemsPerStage = 16u;  // 4 quarters x 4 slices per 128-row tile
    const uint32_t n_items = (uint32_t)args.m_tiles * (uint32_t)kt_n * kItemsPerStage;
    const uint32_t per_group = (uint32_t)kt_n * kItemsPerStage * kGroupM;
#pragma unroll 1
    for (;;) {
      // lane 0 stops taking items once this CTA aborts (broadcast, so the warp stays
      // converged); an item already taken is always finished, so no other CTA's producer
      // waits for an abandoned one
      uint32_t item = 0xFFFFFFFFu;
      if (lane == 0 && *abort_flag == 0) item = atomicAdd(args.work, 1u);
      item = __shfl_sync(0xffffffffu, item, 0);
      if (item >= n_items) break;
      const uint32_t grp = item / per_group;
      const uint32_t r = item - grp * per_group;
      const uint32_t gm = min((uint32_t)kGroupM, (uint32_t)args.m_tiles - grp * kGroupM);
      const uint32_t kc = r / (gm * kItemsPerStage);
      const uint32_t r2 = r - kc * gm * kItemsPerStage;
      const uint32_t mt = grp * kGroupM + r2 / kItemsPerStage;
      const uint32_t sub = r2 % kItemsPerStage;  // quarter = sub / 4, slice = sub % 4
      const uint32_t row_lane = mt * kBM + (sub >> 2) * 32u + (uint32_t)(lane >> 2);
      const uint32_t kb = kc * 16u + (sub & 3u) * 4u + (uint32_t)(lane & 3);
      uint32_t buf[4][8];  // all four blocks of this lane in flight at once
#pragma unroll
      for (uint32_t i = 0; i < 4u; ++i) ld_stream256(args.x + ((int64_t)(row_lane + 8u * i) * cols16 + kb) * 16, buf[i]);
#pragma unroll
      for (uint32_t i = 0; i < 4u; ++i) {
        const uint32_t row = row_lane + 8u * i;
        operand_block<QATF_OPERAND_A>(buf[i], g, (int64_t)row * cols16 + kb, row, kb, atoms_k, true, args.xq_codes,
                                      args.xq_sf, args.xq_deq, args.xq_mask);
      }
      // publish: this lane's stores visible at GPU scope and to the async proxy (the
      // producers' TMA reads), then one release count per warp
      __threadfence();
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __syncwarp();
      if (lane == 0)
        asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(args.ready + (int64_t)mt * kt_n + kc) : "memory");
    }
  };
  if (warp == 0) {
    if (lane == 0) role_producer();
  } else if (warp == 1) {
    if (lane == 0) role_mma();
  } else if (warp >= kEpiFirst && warp < kEpiFirst + EPI) {
    role_epilogue();
  } else if constexpr (FUSE_A) {
    role_quantizer();  // warps 2, 3 and 12..19
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------------- BF16, CTA pairs (cta_group::2)
// A cluster of two CTAs on one TPC computes a 256 x 256 tile with tcgen05.mma.cta_group::2:
// CTA r holds rows [128r, 128r+128) of A and rows [128r, 128r+128) of B's 256 (both in its
// own shared memory at the same offsets); the leader (rank 0) issues the MMAs, each CTA's
// tensor memory receives its own 128 rows of D.  Per CTA and stage only 32 KB cross from L2
// instead of 48 KB.  Both CTAs' loads complete on the leader's `full` barrier, whose one
// arrival is the leader's expect_tx for the bytes of both; the leader's commits reach both
// CTAs' `empty` and `acc_full` barriers; both CTAs' epilogue warps arrive on the leader's
// `acc_empty` barrier.
constexpr int kStages2 = 6;
constexpr int kTileA2 = 128 * kRowBytes;  // 16 KB per CTA and stage
constexpr int kTileB2 = 128 * kRowBytes;  // 16 KB per CTA and stage

struct SmemLayout2 {
  static constexpr int a = 0;
  static constexpr int b = a + kStages2 * kTileA2;
  static constexpr int bars = b + kStages2 * kTileB2;  // full[S], empty[S], acc_full[2], acc_empty[2]
  static constexpr int holder = bars + (2 * kStages2 + 4) * 8;
  static constexpr int flags = holder + 8;
  static constexpr int end = flags + 8;
  static constexpr int bytes = end + 1024;
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Address of the same shared-memory object in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_cta(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// TMA load into this CTA's shared memory whose completion is counted on the pair leader's
// barrier (bar_cluster is a shared::cluster address).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* map, uint32_t bar_cluster, int x,
                                                 int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];" ::"r"(dst),
      "l"(map), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void mma_bf16_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive on the barrier at this shared offset in both CTAs of the pair once the leader's
// earlier tcgen05 operations complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\tmov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          bar)
      : "memory");
}

constexpr uint32_t kIdescPairShape = ((uint32_t)(kBN >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
__host__ __device__ constexpr uint32_t idesc_bf16_pair(bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) | kIdescPairShape;
}

template <bool A_MN, bool B_MN>
__global__ void __launch_bounds__(192, 1)
    tc2_gemm_bf16_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                         const Args args) {
  constexpr int EPI = 4;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  const uint32_t bar_full = s0 + SmemLayout2::bars;
  const uint32_t bar_empty = bar_full + kStages2 * 8;
  const uint32_t bar_acc_full = bar_empty + kStages2 * 8;
  const uint32_t bar_acc_empty = bar_acc_full + 2 * 8;
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + SmemLayout2::holder);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + SmemLayout2::flags);
  constexpr uint32_t kTmemCols = 512u;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int m_pairs = args.m_tiles >> 1;  // 256-row tiles
  const int n_tiles_all = m_pairs * args.n_tiles;
  const int n_total = args.split > 0 ? args.full_units + (n_tiles_all - args.full_units) * args.split : n_tiles_all;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages2; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(bar_acc_full + 8 * b, 1);
      mbar_init(bar_acc_empty + 8 * b, 2 * EPI);
    }
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  fence_before();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival
  fence_after();
  const uint32_t tmem = *holder;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------- producer
    constexpr uint32_t tx = kTileA2 + kTileB2;
    const uint32_t full_leader = map_to_cta(bar_full, 0);
    uint32_t it = 0;
    bool ok = true;
    for (int t = pair; t < n_total && ok; t += n_pairs) {
      const PairUnit U = pair_unit(t, m_pairs, args);
      const int m0 = U.mp * 256 + 128 * (int)rank;
      const int n0 = U.nt * kBN + 128 * (int)rank;
      for (int kt = U.k0; kt < U.k1; ++kt, ++it) {
        const int s = it % kStages2;
        if (!mbar_wait(bar_empty + 8 * s, ((it / kStages2) & 1) ^ 1, abort_flag, args.err)) {
          ok = false;
          break;
        }
        const uint32_t full = full_leader + 8 * s;
        // the leader announces both CTAs' bytes on its own barrier; the peer only loads (a
        // peer refills stage s only after the MMAs consumed it, so no phase is completed early)
        if (rank == 0) mbar_expect_tx(bar_full + 8 * s, 2 * tx);
        const uint32_t sa = s0 + SmemLayout2::a + s * kTileA2;
        const uint32_t sb = s0 + SmemLayout2::b + s * kTileB2;
        if (A_MN) {
          for (int c = 0; c < 2; ++c) tma_load_2d_pair(sa + c * 64 * kRowBytes, &map_a, full, m0 + 64 * c, kt * 64);
        } else {
          tma_load_2d_pair(sa, &map_a, full, kt * 64, m0);
        }
        if (B_MN) {
          for (int c = 0; c < 2; ++c) tma_load_2d_pair(sb + c * 64 * kRowBytes, &map_b, full, n0 + 64 * c, kt * 64);
        } else {
          tma_load_2d_pair(sb, &map_b, full, kt * 64, n0);
        }
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ----------------------------------------------------- MMA issuer (pair leader)
    const uint64_t desc_a0 = A_MN ? smem_desc(s0 + SmemLayout2::a, 64 * kRowBytes, 1024, 2)
                                  : smem_desc(s0 + SmemLayout2::a, 16, 1024, 2);
    const uint64_t desc_b0 = B_MN ? smem_desc(s0 + SmemLayout2::b, 64 * kRowBytes, 1024, 2)
                                  : smem_desc(s0 + SmemLayout2::b, 16, 1024, 2);
    constexpr uint64_t kStepA = A_MN ? 2048 / 16 : 32 / 16;
    constexpr uint64_t kStepB = B_MN ? 2048 / 16 : 32 / 16;
    uint32_t it = 0;
    int li = 0;
    bool ok = true;
    for (int t = pair; t < n_total && ok; t += n_pairs, ++li) {
      const int b = li & 1;
      if (!mbar_wait(bar_acc_empty + 8 * b, ((li >> 1) & 1) ^ 1, abort_flag, args.err)) break;
      fence_after();
      const uint32_t acc = tmem + b * kBN;
      const PairUnit U = pair_unit(t, m_pairs, args);
      for (int kt = U.k0; kt < U.k1; ++kt, ++it) {
        const int s = it % kStages2;
        if (!mbar_wait(bar_full + 8 * s, (it / kStages2) & 1, abort_flag, args.err)) {
          ok = false;
          break;
        }
        fence_after();
        const uint64_t da = desc_a0 + (uint64_t)((s * kTileA2) >> 4);
        const uint64_t db = desc_b0 + (uint64_t)((s * kTileB2) >> 4);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_bf16_pair(acc, da + kStepA * j, db + kStepB * j, idesc_bf16_pair(A_MN, B_MN), (kt != U.k0) || (j != 0));
        mma_commit_pair(bar_empty + 8 * s);
      }
      if (ok) mma_commit_pair(bar_acc_full + 8 * b);
    }
  } else if (warp >= 2) {
    // -------------------------------------------------------------------- epilogue
    const int q = warp & 3;
    const uint32_t acc_empty_leader = map_to_cta(bar_acc_empty, 0);
    int li = 0;
    for (int t = pair; t < n_total; t += n_pairs, ++li) {
      const int b = li & 1;
      if (!mbar_wait(bar_acc_full + 8 * b, (li >> 1) & 1, abort_flag, args.err)) break;
      fence_after();
      const PairUnit U = pair_unit(t, m_pairs, args);
      const int64_t row = (int64_t)U.mp * 256 + 128 * rank + 32 * q + lane;
      const int64_t col0 = (int64_t)U.nt * kBN;
      __nv_bfloat16* orow = args.out + row * args.ldo + col0;
      const uint32_t tbase = tmem + b * kBN + ((uint32_t)(32 * q) << 16);
#pragma unroll 1
      for (int c = 0; c < kBN / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + 32 * c, r);
        if (c == kBN / 32 - 1) {
          fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_remote(acc_empty_leader + 8 * b);
        }
        if (U.part >= 0) {
          // a K-slice of a tail tile: its FP32 partial sums go to the workspace
          float* wrow = args.ws + ((int64_t)U.part * 256 + 128 * rank + 32 * q + lane) * 256 + 32 * c;
#pragma unroll
          for (int v = 0; v < 4; ++v) st256(wrow + 8 * v, r + 8 * v);
          continue;
        }
        uint32_t keep = 0xFFFFFFFFu;
        if (args.mask != nullptr) keep = *reinterpret_cast<const uint32_t*>(args.mask + (row * args.ldo + col0 + 32 * c) / 8);
        uint32_t o[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          uint32_t v = pack_bf16x2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
          if (!((keep >> (2 * i)) & 1u)) v &= 0xFFFF0000u;
          if (!((keep >> (2 * i + 1)) & 1u)) v &= 0x0000FFFFu;
          o[i] = v;
        }
        st256(orow + 32 * c, o);
        st256(orow + 32 * c + 16, o + 8);
      }
    }
  }
  fence_before();
  cluster_sync();  // no CTA leaves while its peer may still arrive on its barriers or use its TMEM
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ------------------------------------------------------- FP4, CTA pairs (cta_group::2)
// The block-scaled FP4 GEMM (NVFP4 or MXFP4) on 256 x 256 tiles of a CTA pair, with the
// protocol of the BF16 pair kernel above: CTA r loads rows [128r, 128r + 128) of A's tile and of
// B's, so per MMA each SM reads 8 KB of operands from its shared memory instead of 12 KB; both
// CTAs also load, at the same shared offsets, the scale blocks of their own 128 rows of A and
// of all 256 rows of B (B's scales are needed in both CTAs' tensor memory), all counted on the
// leader's `full` barrier.  The leader issues tcgen05.cp.cta_group::2 (each CTA's blocks into its
// own tensor memory) and the M = 256 MMAs; one accumulator per CTA (256 columns beside the 48
// of scales), drained by eight epilogue warps per CTA into registers before it is handed back.
template <int KIND>
struct SmemLayoutP {
  static constexpr int stages = KIND == kNVF4 ? 3 : 4;
  static constexpr int sfa_bytes = SmemLayout<KIND>::sfa_bytes;
  static constexpr int sfb_bytes = SmemLayout<KIND>::sfb_bytes;
  static constexpr int a = 0;
  static constexpr int b = a + stages * kTileA2;
  static constexpr int sfa = b + stages * kTileB2;
  static constexpr int sfb = sfa + stages * sfa_bytes;
  static constexpr int bars = sfb + stages * sfb_bytes;  // full[S], empty[S], acc_full, acc_empty
  static constexpr int holder = bars + (2 * stages + 2) * 8;
  static constexpr int flags = holder + 8;
  static constexpr int end = flags + 8;
  static constexpr int bytes = end + 1024;
};

__device__ __forceinline__ void sf_copy_wide_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.128x256b [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

template <int KIND>
__device__ __forceinline__ void mma_fp4_pair(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t sfa,
                                             uint32_t sfb, uint32_t acc) {
  if constexpr (KIND == kNVF4) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(acc), "r"(sfa), "r"(sfb)
        : "memory");
  }
}

// Instruction descriptors of the pair MMAs (M = 256): as the single-CTA ones, other shape.
__host__ __device__ constexpr uint32_t idesc_fp4_pair(int kind, uint32_t sf_id) {
  return (1u << 7) | (1u << 10) | (kind == kMXF4 ? (1u << 23) | (sf_id << 29) | (sf_id << 4) : 0u) |
         kIdescPairShape;
}

template <int KIND>
__global__ void __launch_bounds__(64 + 32 * 8, 1)
    tc2_gemm_fp4_kernel(const __grid_constant__ CUtensorMap map_a, const __grid_constant__ CUtensorMap map_b,
                        const __grid_constant__ CUtensorMap map_sfa, const __grid_constant__ CUtensorMap map_sfb,
                        const Args args) {
  using L = SmemLayoutP<KIND>;
  constexpr int kStages = L::stages;
  constexpr int EPI = 8;
  constexpr int kColsPerWarp = kBN * 4 / EPI;  // 128
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t s0 = smem_u32(smem);
  const uint32_t bar_full = s0 + L::bars;
  const uint32_t bar_empty = bar_full + kStages * 8;
  const uint32_t bar_acc_full = bar_empty + kStages * 8;
  const uint32_t bar_acc_empty = bar_acc_full + 8;
  uint32_t* holder = reinterpret_cast<uint32_t*>(smem + L::holder);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + L::flags);
  constexpr uint32_t kTmemCols = 512u;
  constexpr uint32_t kSfaCol = kBN;           // 16 columns: 4 K-blocks x 4
  constexpr uint32_t kSfbCol = kSfaCol + 16;  // 32 columns: 4 K-blocks x 8
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1;
  const int n_pairs = gridDim.x >> 1;
  const int m_pairs = args.m_tiles >> 1;  // 256-row tiles
  const int n_total = m_pairs * args.n_tiles;
  const int kt_n = args.k_tiles;

  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(bar_full + 8 * s, 1);
      mbar_init(bar_empty + 8 * s, 1);
    }
    mbar_init(bar_acc_full, 1);
    mbar_init(bar_acc_empty, 2 * EPI);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  fence_before();
  cluster_sync();  // both CTAs' barriers exist before any remote arrival
  fence_after();
  const uint32_t tmem = *holder;

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------------------- producer
    constexpr uint32_t tx = kTileA2 + kTileB2 + L::sfa_bytes + L::sfb_bytes;
    const uint32_t full_leader = map_to_cta(bar_full, 0);
    uint32_t it = 0;
    bool ok = true;
    for (int t = pair; t < n_total && ok; t += n_pairs) {
      int mp, nt;
      tile_coords(t, m_pairs, args.n_tiles, mp, nt);
      const int mt = 2 * mp + (int)rank;  // this CTA's 128-row tile
      const int m0 = mt * 128;
      const int n0 = nt * kBN + 128 * (int)rank;
      for (int kt = 0; kt < kt_n; ++kt, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(bar_empty + 8 * s, ((it / kStages) & 1) ^ 1, abort_flag, args.err)) {
          ok = false;
          break;
        }
        const uint32_t full = full_leader + 8 * s;
        // the leader announces both CTAs' bytes on its own barrier; the peer only loads
        if (rank == 0) mbar_expect_tx(bar_full + 8 * s, 2 * tx);
        tma_load_2d_pair(s0 + L::a + s * kTileA2, &map_a, full, kt * 128, m0);
        tma_load_2d_pair(s0 + L::b + s * kTileB2, &map_b, full, kt * 128, n0);
        tma_load_2d_pair(s0 + L::sfa + s * L::sfa_bytes, &map_sfa, full, 0,
                         (int)(((int64_t)mt * kt_n + kt) * (L::sfa_bytes / 256)));
        tma_load_2d_pair(s0 + L::sfb + s * L::sfb_bytes, &map_sfb, full, 0,
                         (int)(((int64_t)nt * kt_n + kt) * (L::sfb_bytes / 256)));
      }
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // ----------------------------------------------------- MMA issuer (pair leader)
    const uint64_t desc_a0 = smem_desc(s0 + L::a, 16, 1024, 2);
    const uint64_t desc_b0 = smem_desc(s0 + L::b, 16, 1024, 2);
    uint32_t it = 0;
    int li = 0;
    bool ok = true;
    for (int t = pair; t < n_total && ok; t += n_pairs, ++li) {
      if (!mbar_wait(bar_acc_empty, (li & 1) ^ 1, abort_flag, args.err)) break;
      fence_after();
      for (int kt = 0; kt < kt_n; ++kt, ++it) {
        const int s = it % kStages;
        if (!mbar_wait(bar_full + 8 * s, (it / kStages) & 1, abort_flag, args.err)) {
          ok = false;
          break;
        }
        fence_after();
        const uint32_t ssa = s0 + L::sfa + s * L::sfa_bytes;
        const uint32_t ssb = s0 + L::sfb + s * L::sfb_bytes;
        const uint64_t da = desc_a0 + (uint64_t)((s * kTileA2) >> 4);
        const uint64_t db = desc_b0 + (uint64_t)((s * kTileB2) >> 4);
        if constexpr (KIND == kNVF4) {
#pragma unroll
          for (int h = 0; h < 2; ++h) sf_copy_wide_pair(tmem + kSfaCol + 8 * h, smem_desc(ssa + 4096 * h, 128, 256, 0));
#pragma unroll
          for (int j = 0; j < 4; ++j) sf_copy_wide_pair(tmem + kSfbCol + 8 * j, smem_desc(ssb + 4096 * j, 128, 256, 0));
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_fp4_pair<KIND>(tmem, da + 2 * j, db + 2 * j, idesc_fp4_pair(KIND, 0), tmem + kSfaCol + 4 * j,
                               tmem + kSfbCol + 8 * j, (kt | j) != 0);
        } else {
          sf_copy_wide_pair(tmem + kSfaCol, smem_desc(ssa, 128, 256, 0));
#pragma unroll
          for (int h = 0; h < 2; ++h) sf_copy_wide_pair(tmem + kSfbCol + 8 * h, smem_desc(ssb + 4096 * h, 128, 256, 0));
#pragma unroll
          for (int j = 0; j < 4; ++j)
            mma_fp4_pair<KIND>(tmem, da + 2 * j, db + 2 * j, idesc_fp4_pair(KIND, 2u * (j & 1)),
                               tmem + kSfaCol + 4 * (j >> 1), tmem + kSfbCol + 8 * (j >> 1), (kt | j) != 0);
        }
        mma_commit_pair(bar_empty + 8 * s);
      }
      if (ok) mma_commit_pair(bar_acc_full);
    }
  } else if (warp >= 2) {
    // -------------------------------------------------------------------- epilogue
    const int e = warp - 2;
    const int q = warp & 3;                     // TMEM lane quarter this warp may read
    const int c_base = (e / 4) * kColsPerWarp;  // its column range
    float alpha = 1.0f;
    if constexpr (KIND == kNVF4) alpha = __fdiv_rn(args.a_amax[0], 2688.0f) * __fdiv_rn(args.b_amax[0], 2688.0f);
    const uint32_t acc_empty_leader = map_to_cta(bar_acc_empty, 0);
    int li = 0;
    for (int t = pair; t < n_total; t += n_pairs, ++li) {
      if (!mbar_wait(bar_acc_full, li & 1, abort_flag, args.err)) break;
      fence_after();
      int mp, nt;
      tile_coords(t, m_pairs, args.n_tiles, mp, nt);
      const int64_t row = (int64_t)mp * 256 + 128 * rank + 32 * q + lane;
      const int64_t col0 = (int64_t)nt * kBN + c_base;
      __nv_bfloat16* orow = args.out + row * args.ldo + col0;
      const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + c_base;
      // the whole column range into registers as BF16 pairs, then the accumulator back
      uint32_t o[kColsPerWarp / 32][16];
#pragma unroll
      for (int c = 0; c < kColsPerWarp / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(tbase + 32 * c, r);
#pragma unroll
        for (int i = 0; i < 16; ++i)
          o[c][i] = pack_bf16x2(__uint_as_float(r[2 * i]) * alpha, __uint_as_float(r[2 * i + 1]) * alpha);
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc_empty_leader);
#pragma unroll
      for (int c = 0; c < kColsPerWarp / 32; ++c) {
        st256(orow + 32 * c, o[c]);
        st256(orow + 32 * c + 16, o[c] + 8);
      }
    }
  }
  fence_before();
  cluster_sync();  // no CTA leaves while its peer may still arrive on its barriers or use its TMEM
  if (warp == 1) {
    fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// Sum of the K-slices of each split tail tile (in slice order), then the STE mask and the BF16
// store of the whole-tile epilogue: thread = 8 consecutive columns of one row of one tile.
__global__ void __launch_bounds__(256) splitk_reduce_kernel(const float* __restrict__ ws, int tail, int split,
                                                            int full_units, int m_pairs, int n_tiles,
                                                            __nv_bfloat16* __restrict__ out, int64_t ldo,
                                                            const uint8_t* __restrict__ mask) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)tail * 256 * 32) return;
  const int cg = (int)(idx & 31);
  const int row = (int)((idx >> 5) & 255);
  const int t = (int)(idx >> 13);
  int mp, nt;
  tile_coords(full_units + t, m_pairs, n_tiles, mp, nt);
  float acc[8];
  const float* p = ws + ((int64_t)t * split * 256 + row) * 256 + cg * 8;
  {
    const float4 v0 = *reinterpret_cast<const float4*>(p);
    const float4 v1 = *reinterpret_cast<const float4*>(p + 4);
    acc[0] = v0.x; acc[1] = v0.y; acc[2] = v0.z; acc[3] = v0.w;
    acc[4] = v1.x; acc[5] = v1.y; acc[6] = v1.z; acc[7] = v1.w;
  }
  for (int sl = 1; sl < split; ++sl) {
    const float* q = p + (int64_t)sl * 256 * 256;
    const float4 v0 = *reinterpret_cast<const float4*>(q);
    const float4 v1 = *reinterpret_cast<const float4*>(q + 4);
    acc[0] += v0.x; acc[1] += v0.y; acc[2] += v0.z; acc[3] += v0.w;
    acc[4] += v1.x; acc[5] += v1.y; acc[6] += v1.z; acc[7] += v1.w;
  }
  const int64_t grow = (int64_t)mp * 256 + row;
  const int64_t gcol = (int64_t)nt * 256 + cg * 8;
  uint32_t keep = 0xFFu;
  if (mask != nullptr) keep = mask[(grow * ldo + gcol) >> 3];
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    uint32_t v = pack_bf16x2(acc[2 * i], acc[2 * i + 1]);
    if (!((keep >> (2 * i)) & 1u)) v &= 0xFFFF0000u;
    if (!((keep >> (2 * i + 1)) & 1u)) v &= 0x0000FFFFu;
    o[i] = v;
  }
  *reinterpret_cast<uint4*>(out + grow * ldo + gcol) = make_uint4(o[0], o[1], o[2], o[3]);
}

// ------------------------------------------------------------------------------- host
// Row-major [outer, inner] matrix, box [box_outer, box_inner], 128-byte swizzle.
bool make_map(CUtensorMap* map, const void* base, CUtensorMapDataType dt, int elem_bytes, uint64_t inner,
              uint64_t outer, uint32_t box_inner, uint32_t box_outer) {
  return make_map_2d(map, base, dt, elem_bytes, inner, outer, box_inner, box_outer);
}

template <typename Kernel, typename... P>
int launch_cluster2(Kernel k, int threads, int smem_bytes, int64_t pairs, cudaStream_t s, P... params) {
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes) != cudaSuccess)
    return QATF_ERR_LAUNCH;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3((unsigned)threads);
  cfg.dynamicSmemBytes = (size_t)smem_bytes;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  // a persistent grid must be co-resident: not every SM pairs up into a cluster (GPC sizes)
  cfg.gridDim = dim3((unsigned)(2 * (num_sms() / 2)));
  int clusters = 0;
  if (cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) != cudaSuccess || clusters <= 0) return QATF_ERR_LAUNCH;
  cfg.gridDim = dim3((unsigned)(2 * std::min<int64_t>(pairs, clusters)));
  if (cudaLaunchKernelEx(&cfg, k, params...) != cudaSuccess) return launched(QATF_ERR_LAUNCH);
  return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
}

template <int KIND, bool A_MN, bool B_MN>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, Args args, int64_t m, int64_t n, cudaStream_t s) {
  constexpr int NACC = is_fp4(KIND) ? 1 : 2;
  constexpr int EPI = is_fp4(KIND) ? 8 : 4;
  auto k = tc_gemm_kernel<KIND, A_MN, B_MN, NACC, EPI>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemLayout<KIND>::bytes) != cudaSuccess)
    return QATF_ERR_LAUNCH;
  args.m_tiles = (int)(m / kBM);
  args.n_tiles = (int)(n / kBN);
  const int64_t tiles = (int64_t)args.m_tiles * args.n_tiles;
  const int grid = (int)std::min<int64_t>(tiles, num_sms());
  k<<<grid, 64 + 32 * EPI, SmemLayout<KIND>::bytes, s>>>(ma, mb, args);
  return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
}

// Which FP4 GEMMs with M % 256 == 0 run on CTA pairs.  Measured at the benchmark shapes, one
// box, alternating builds: MXFP4 (configuration 2, [16384, 4096] x [24576, 4096]) 712 us on
// pairs against 805 on single CTAs; NVFP4 (configuration 4) 231 against 222, as the leader
// then issues both CTAs' six scale copies per stage (MXFP4 has three), so NVFP4 stays on single
// CTAs unless built with QATF_NVFP4_PAIR=1.
#ifndef QATF_MXFP4_PAIR
#define QATF_MXFP4_PAIR 1
#endif
#ifndef QATF_NVFP4_PAIR
#define QATF_NVFP4_PAIR 0
#endif
template <int KIND>
int launch_fp4_pair(const uint8_t* a_codes, const uint8_t* a_scales, const uint8_t* b_codes, const uint8_t* b_scales,
                    Args args, int64_t m, int64_t n, int64_t k, cudaStream_t s) {
  using L = SmemLayoutP<KIND>;
  const int64_t per_elt_div = KIND == kNVF4 ? 4 : 8;  // scale bytes: 4 copies of 1 byte per 16 / 32 elements
  CUtensorMap ma, mb, msa, msb;
  if (!make_map(&ma, a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)m, 128, 128) ||
      !make_map(&mb, b_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)n, 128, 128) ||
      !make_map_2d_plain(&msa, a_scales, 256, (uint64_t)(m * k / per_elt_div / 256), L::sfa_bytes / 256) ||
      !make_map_2d_plain(&msb, b_scales, 256, (uint64_t)(n * k / per_elt_div / 256), L::sfb_bytes / 256))
    return QATF_ERR_LAUNCH;
  args.m_tiles = (int)(m / kBM);
  args.n_tiles = (int)(n / kBN);
  const int64_t units = (m / 256) * (n / kBN);
  return launch_cluster2(tc2_gemm_fp4_kernel<KIND>, 64 + 32 * 8, L::bytes, units, s, ma, mb, msa, msb, args);
}

// W4A4 forward with the activation quantized inside the FP4 GEMM kernel (FUSE_A).
int launch_fused(const CUtensorMap& ma, const CUtensorMap& mb, Args args, int64_t m, int64_t n, cudaStream_t s) {
  auto k = tc_gemm_kernel<kNVF4, false, false, 1, 8, true>;
  if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemLayout<kNVF4>::bytes) != cudaSuccess)
    return QATF_ERR_LAUNCH;
  args.m_tiles = (int)(m / kBM);
  args.n_tiles = (int)(n / kBN);
  const int64_t tiles = (int64_t)args.m_tiles * args.n_tiles;
  const int grid = (int)std::min<int64_t>(tiles, num_sms());
  k<<<grid, kFusedThreads, SmemLayout<kNVF4>::bytes, s>>>(ma, mb, args);
  return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
}

// Co-resident CTA pairs of the pair kernel on the current device (the same for every
// instantiation: same block size and shared memory); 0 on error.
int pair_slots() {
  static std::mutex mu;
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
  std::lock_guard<std::mutex> lock(mu);
  if (cached[dev] == 0) {
    auto k = tc2_gemm_bf16_kernel<false, false>;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, SmemLayout2::bytes) != cudaSuccess)
      return 0;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(192u);
    cfg.dynamicSmemBytes = (size_t)SmemLayout2::bytes;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cfg.gridDim = dim3((unsigned)(2 * (num_sms() / 2)));
    int clusters = 0;
    if (cudaOccupancyMaxActiveClusters(&clusters, k, &cfg) != cudaSuccess || clusters <= 0) return 0;
    cached[dev] = clusters;
  }
  return cached[dev];
}

// Split-K of the last wave: when the pair tiles leave a last wave less than half full, each of
// its `tail` tiles is cut into `split` K-slices (at least four 64-column K tiles each) so the
// slices fill the wave; they write FP32 partial tiles to a workspace that a second kernel sums.
struct SplitPlan {
  int split = 0;
  int full_units = 0;
  int64_t units = 0;
  int64_t ws_bytes = 0;
};

SplitPlan plan_split(int64_t m, int64_t n, int64_t k, int slots) {
  SplitPlan p;
  const int64_t tiles = (m / 256) * (n / kBN);
  p.full_units = (int)tiles;
  p.units = tiles;
  const int64_t tail = slots > 0 ? tiles % slots : 0;
  if (slots <= 0 || tiles <= slots || tail == 0 || 2 * tail > slots) return p;
  const int64_t split = std::min<int64_t>(slots / tail, (k / 64) / 4);
  if (split < 2) return p;
  p.split = (int)split;
  p.full_units = (int)(tiles - tail);
  p.units = (tiles - tail) + tail * split;
  p.ws_bytes = tail * split * 256 * 256 * (int64_t)sizeof(float);
  return p;
}

template <bool A_MN, bool B_MN>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, Args args, int64_t m, int64_t n, int64_t k,
                void* workspace, int64_t workspace_bytes, cudaStream_t s) {
  args.m_tiles = (int)(m / kBM);
  args.n_tiles = (int)(n / kBN);
  const SplitPlan plan = plan_split(m, n, k, pair_slots());
  int64_t units = (int64_t)(args.m_tiles / 2) * args.n_tiles;
  args.split = 0;
  if (plan.split > 0 && workspace != nullptr && workspace_bytes >= plan.ws_bytes && aligned32(workspace)) {
    args.split = plan.split;
    args.full_units = plan.full_units;
    args.ws = static_cast<float*>(workspace);
    units = plan.units;
  }
  const int st = launch_cluster2(tc2_gemm_bf16_kernel<A_MN, B_MN>, 192, SmemLayout2::bytes, units, s, ma, mb, args);
  if (st != QATF_OK || args.split == 0) return st;
  const int tail = (int)((int64_t)(args.m_tiles / 2) * args.n_tiles - args.full_units);
  const int64_t threads = (int64_t)tail * 256 * 32;
  splitk_reduce_kernel<<<(unsigned)((threads + 255) / 256), 256, 0, s>>>(
      args.ws, tail, args.split, args.full_units, args.m_tiles / 2, args.n_tiles, args.out, args.ldo, args.mask);
  return launched(cudaGetLastError() == cudaSuccess ? QATF_OK : QATF_ERR_LAUNCH);
}

// sm_100 check.  Also makes the device's primary context current on the calling thread: the
// tensor maps are encoded through the driver API, which needs one, and a thread whose first
// CUDA work is this call (an autograd backward thread, say) has none yet.
bool device_ok() {
  int dev = 0, major = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || cudaSetDevice(dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  return major == 10;
}

}  // namespace tc
}  // namespace qatf

using namespace qatf;
using namespace qatf::tc;

// The kernels number output tiles (128 x 256) with 32-bit ints: larger grids are refused.
static inline bool tiles_fit(int64_t m, int64_t n) { return (m / kBM) * (n / kBN) <= (int64_t)INT32_MAX; }

extern "C" int qatf_nvfp4_gemm(const uint8_t* a_codes, const uint8_t* a_scales, const float* a_amax,
                               const uint8_t* b_codes, const uint8_t* b_scales, const float* b_amax, int64_t m,
                               int64_t n, int64_t k, void* out, int* err, void* stream) {
  if (m < 0 || n < 0 || k < 0) return QATF_ERR_INVALID;
  if (m % kBM || n % kBN || k % 256) return QATF_ERR_UNSUPPORTED;
  if (m > (int64_t)kBM * 65535 || k > (1 << 30) || n > (1 << 30) || !tiles_fit(m, n)) return QATF_ERR_UNSUPPORTED;
  if (m == 0 || n == 0) return QATF_OK;
  if (!a_codes || !a_scales || !a_amax || !b_codes || !b_scales || !b_amax || !out || !err) return QATF_ERR_INVALID;
  if (!aligned16(a_codes) || !aligned16(b_codes) || !aligned16(a_scales) || !aligned16(b_scales) || !aligned16(out))
    return QATF_ERR_INVALID;
  if (!device_ok()) return QATF_ERR_DEVICE;
  CUtensorMap ma, mb;
  if (!make_map(&ma, a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)m, 128, kBM) ||
      !make_map(&mb, b_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)n, 128, kBN))
    return QATF_ERR_LAUNCH;
  Args args{};
  args.k_tiles = (int)(k / 256);
  args.sfa = a_scales;
  args.sfb = b_scales;
  args.a_amax = a_amax;
  args.b_amax = b_amax;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.ldo = n;
  args.mask = nullptr;
  args.err = err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#if QATF_NVFP4_PAIR
  if (m % 256 == 0) return launch_fp4_pair<kNVF4>(a_codes, a_scales, b_codes, b_scales, args, m, n, k, s);
#endif
  return launch<kNVF4, false, false>(ma, mb, args, m, n, s);
}

extern "C" int qatf_mxfp4_gemm(const uint8_t* a_codes, const uint8_t* a_scales, const uint8_t* b_codes,
                               const uint8_t* b_scales, int64_t m, int64_t n, int64_t k, void* out, int* err,
                               void* stream) {
  if (m < 0 || n < 0 || k < 0) return QATF_ERR_INVALID;
  if (m % kBM || n % kBN || k % 256) return QATF_ERR_UNSUPPORTED;
  if (m > (int64_t)kBM * 65535 || k > (1 << 30) || n > (1 << 30) || !tiles_fit(m, n)) return QATF_ERR_UNSUPPORTED;
  if (m == 0 || n == 0) return QATF_OK;
  if (!a_codes || !a_scales || !b_codes || !b_scales || !out || !err) return QATF_ERR_INVALID;
  if (!aligned16(a_codes) || !aligned16(b_codes) || !aligned16(a_scales) || !aligned16(b_scales) || !aligned16(out))
    return QATF_ERR_INVALID;
  if (!device_ok()) return QATF_ERR_DEVICE;
  CUtensorMap ma, mb;
  if (!make_map(&ma, a_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)m, 128, kBM) ||
      !make_map(&mb, b_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)n, 128, kBN))
    return QATF_ERR_LAUNCH;
  Args args{};
  args.k_tiles = (int)(k / 256);
  args.sfa = a_scales;
  args.sfb = b_scales;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.ldo = n;
  args.mask = nullptr;
  args.err = err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#if QATF_MXFP4_PAIR
  if (m % 256 == 0) return launch_fp4_pair<kMXF4>(a_codes, a_scales, b_codes, b_scales, args, m, n, k, s);
#endif
  return launch<kMXF4, false, false>(ma, mb, args, m, n, s);
}

extern "C" int qatf_nvfp4_linear_fwd(const void* x, const float* x_amax, const uint8_t* w_codes,
                                     const uint8_t* w_scales, const float* w_amax, int64_t m, int64_t n, int64_t k,
                                     uint8_t* x_codes, uint8_t* x_scales, void* x_deq, uint8_t* x_mask,
                                     uint32_t* sync, void* out, int* err, void* stream) {
  if (m < 0 || n < 0 || k < 0) return QATF_ERR_INVALID;
  if (m % kBM || n % kBN || k % 256) return QATF_ERR_UNSUPPORTED;
  if (m > (int64_t)kBM * 65535 || k > (1 << 30) || n > (1 << 30) || !tiles_fit(m, n) ||
      m * (k / 16) >= (int64_t(1) << 32))
    return QATF_ERR_UNSUPPORTED;
  if (m == 0 || n == 0) return QATF_OK;
  if (!x || !x_amax || !w_codes || !w_scales || !w_amax || !x_codes || !x_scales || !sync || !out || !err)
    return QATF_ERR_INVALID;
  if (!aligned32(x) || !aligned16(w_codes) || !aligned16(w_scales) || !aligned16(x_codes) || !aligned16(x_scales) ||
      !aligned16(out) || (x_deq != nullptr && !aligned32(x_deq)) || (x_mask != nullptr && !aligned16(x_mask)) ||
      (reinterpret_cast<uintptr_t>(sync) & 3u) != 0)
    return QATF_ERR_INVALID;
  if (!device_ok()) return QATF_ERR_DEVICE;
  CUtensorMap ma, mb;
  if (!make_map(&ma, x_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)m, 128, kBM) ||
      !make_map(&mb, w_codes, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)k / 2, (uint64_t)n, 128, kBN))
    return QATF_ERR_LAUNCH;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int64_t k_tiles = k / 256;
  if (cudaMemsetAsync(sync, 0, (size_t)QATF_NVFP4_LINEAR_SYNC_WORDS(m, k) * sizeof(uint32_t), s) != cudaSuccess)
    return QATF_ERR_LAUNCH;
  Args args{};
  args.k_tiles = (int)k_tiles;
  args.sfa = x_scales;
  args.sfb = w_scales;
  args.a_amax = x_amax;
  args.b_amax = w_amax;
  args.out = static_cast<__nv_bfloat16*>(out);
  args.ldo = n;
  args.mask = nullptr;
  args.err = err;
  args.x = static_cast<const __nv_bfloat16*>(x);
  args.xq_codes = x_codes;
  args.xq_sf = x_scales;
  args.xq_deq = static_cast<__nv_bfloat16*>(x_deq);
  args.xq_mask = x_mask;
  args.ready = sync;
  args.work = sync + (m / kBM) * k_tiles;
  return launch_fused(ma, mb, args, m, n, s);
}

extern "C" int64_t qatf_bf16_gemm_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m <= 0 || n <= 0 || k <= 0 || m % 256 || n % kBN || k % 64) return 0;
  if (!device_ok()) return 0;
  return plan_split(m, n, k, pair_slots()).ws_bytes;
}

extern "C" int qatf_bf16_gemm(const void* a, int a_layout, const void* b, int b_layout, int64_t m, int64_t n,
                              int64_t k, const uint8_t* mask_bits, void* out, int* err, void* stream) {
  return qatf_bf16_gemm_ws(a, a_layout, b, b_layout, m, n, k, mask_bits, out, err, nullptr, 0, stream);
}

extern "C" int qatf_bf16_gemm_ws(const void* a, int a_layout, const void* b, int b_layout, int64_t m, int64_t n,
                                 int64_t k, const uint8_t* mask_bits, void* out, int* err, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  if (m < 0 || n < 0 || k < 0) return QATF_ERR_INVALID;
  if ((a_layout != QATF_K_MAJOR && a_layout != QATF_MN_MAJOR) || (b_layout != QATF_K_MAJOR && b_layout != QATF_MN_MAJOR))
    return QATF_ERR_INVALID;
  if (m % kBM || n % kBN || k % 64) return QATF_ERR_UNSUPPORTED;
  if (m > (int64_t)kBM * 65535 || k > (1 << 30) || n > (1 << 30) || !tiles_fit(m, n)) return QATF_ERR_UNSUPPORTED;
  if (m == 0 || n == 0) return QATF_OK;
  if (!a || !b || !out || !err || !aligned16(a) || !aligned16(b) || !aligned16(out)) return QATF_ERR_INVALID;
  if (mask_bits != nullptr && !aligned16(mask_bits)) return QATF_ERR_INVALID;
  if (!device_ok()) return QATF_ERR_DEVICE;
  const bool a_mn = a_layout == QATF_MN_MAJOR;
  const bool b_mn = b_layout == QATF_MN_MAJOR;
  // CTA pairs (256-row tiles) when M allows; each CTA then loads 128 rows of B per stage
  const bool pair = m % 256 == 0 && num_sms() >= 2;
  const uint32_t b_rows = pair ? 128u : (uint32_t)kBN;
  CUtensorMap ma, mb;
  const bool ok_a = a_mn ? make_map(&ma, a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)m, (uint64_t)k, 64, 64)
                         : make_map(&ma, a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)k, (uint64_t)m, 64, kBM);
  const bool ok_b = b_mn ? make_map(&mb, b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)n, (uint64_t)k, 64, 64)
                         : make_map(&mb, b, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, (uint64_t)k, (uint64_t)n, 64, b_rows);
  if (!ok_a || !ok_b) return QATF_ERR_LAUNCH;
  Args args{};
  args.k_tiles = (int)(k / 64);
  args.out = static_cast<__nv_bfloat16*>(out);
  args.ldo = n;
  args.mask = mask_bits;
  args.err = err;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (pair) {
    if (!a_mn && !b_mn) return launch_pair<false, false>(ma, mb, args, m, n, k, workspace, workspace_bytes, s);
    if (!a_mn && b_mn) return launch_pair<false, true>(ma, mb, args, m, n, k, workspace, workspace_bytes, s);
    if (a_mn && !b_mn) return launch_pair<true, false>(ma, mb, args, m, n, k, workspace, workspace_bytes, s);
    return launch_pair<true, true>(ma, mb, args, m, n, k, workspace, workspace_bytes, s);
  }
  if (!a_mn && !b_mn) return launch<kKindBF16, false, false>(ma, mb, args, m, n, s);
  if (!a_mn && b_mn) return launch<kKindBF16, false, true>(ma, mb, args, m, n, s);
  if (a_mn && !b_mn) return launch<kKindBF16, true, false>(ma, mb, args, m, n, s);
  return launch<kKindBF16, true, true>(ma, mb, args, m, n, s);
}
