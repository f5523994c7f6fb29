// gemm_tc.cu -- K2: W8A8 GEMM on the 5th-generation tensor cores (sm_100a).
//
//   acc[m,n] = sum_k A[m,k] * B[n,k]                   int8 x int8 -> int32 (TMEM)
//   out[m,n] = ((f32(acc) * sa[m|0]) * sb[n]) + bias[n]  fp32 epilogue -> out dtype
//
// Replaces quantization/w8a8_triton_kernels.py:174-318 (_w8a8_scaled_mm[_nomask]_kernel),
// :67-171 (_int8_mm_no_scale[_nomask]_kernel) and kernels/quantization.py:38-105
// (_w8a8_matmul_kernel).  The epilogue performs the reference's fp32 steps one
// rounded op at a time, so int32 accumulators and the scaled outputs are
// bit-identical to the reference's arithmetic.
//
// Design (one CTA per SM, persistent over 128x256 output tiles):
//   warp 0      TMA producer: 128-byte-swizzled A[128x128B] and B[256x128B]
//               tiles into a 4-stage shared-memory ring (48 KB per stage);
//               A is streamed with an L2 evict-first policy, B (the 7.3 MB
//               weight, reused by every tile) with evict-last.
//   warp 1      MMA issuer: allocates 512 TMEM columns (two 128x256 int32
//               accumulators), issues tcgen05.mma.cta_group::1.kind::i8
//               (M=128, N=256, K=32) from one thread, frees ring slots with
//               tcgen05.commit -> mbarrier.
//   warps 2-5   epilogue: tcgen05.ld 32x32b of the finished accumulator,
//               dequant + bias in fp32, vector stores; releases the TMEM
//               buffer so the MMA warp overlaps the next tile's main loop.
// For M >= RB_GEMM_PAIR_MIN_M a two-SM variant (namespace pair) runs each
// 256x256 tile on a cluster of two CTAs with tcgen05.mma.cta_group::2; with
// fewer tiles than half the pairs (from M = RB_GEMM_PAIR_SPLIT_MIN_M when the
// caller gives a workspace) it splits each tile's K range over pairs, and for
// smaller M with fewer tiles than SMs the one-SM kernel splits K across CTAs;
// both write int32 partials that splitk_finalize_kernel sums; for
// M <= 16 w8a8_gemv_kernel uses dp4a on the CUDA cores in clusters of 8 CTAs
// split along K, whose partial sums meet in the leader's shared memory.  No
// TMA load carries a cluster multicast (only tcgen05.commit signals both CTAs
// of a pair).  Every mbarrier
// wait is bounded (common.cuh): on timeout the kernel records a watchdog code,
// drains what it issued and returns instead of hanging.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"

// smallest M that uses the two-SM kernel.  Per SM a pair tile loads a third
// fewer operand bytes per MMA than a one-SM tile, and from M = 4096 (16 row
// blocks of 256, 32 pairs) that outweighs the idle SMs: at K = 14336, N = 512
// on a B200 it takes 57 / 57 / 59 / 90 us at M = 4096 / 6144 / 8192 / 12288
// against 58 / 64 / 66 / 103 us for the split one-SM kernel.  Below it the
// one-SM kernel, split along K, spreads the work over all SMs.
#ifndef RB_GEMM_PAIR_MIN_M
#define RB_GEMM_PAIR_MIN_M 4096
#endif
// With a split-K workspace the two-SM kernel takes over from M = 2048: its
// 256 x 256 tiles split along K over the pairs beat the split one-SM kernel
// (K = 14336, N = 512 on a B200: M = 2048 / 3072 / 4096 in 24.9 / 30.3 /
// 34.5 us against 25.9 / 31.7 us split one-SM and 43.5 us unsplit pairs; at
// M = 1024 the one-SM split is ahead, 20.5 against 20.9 us).
#ifndef RB_GEMM_PAIR_SPLIT_MIN_M
#define RB_GEMM_PAIR_SPLIT_MIN_M 2048
#endif
// M range of the swapped-operand cluster kernel (the weight as the MMA's 128-row
// operand, the activation rows as its N, K split over a 16-CTA cluster).  Its
// fixed cost (cluster launch, TMEM, two cluster barriers, the DSMEM sum) is
// several us on a B200, so the dp4a GEMV keeps M <= RB_GEMV_MAX_M; up to 256
// rows (the MMA's largest N) it beats the split one-SM kernel (K = 14336,
// N = 512: M = 17 / 64 / 128 / 192 / 256 take 7.4 / 8.5 / 10.6 / 12.7 / 14.6 us
// against 10.8 / 12.0 / 14.5 / 14.9 / 15.2 us split).
#ifndef RB_GEMV_MAX_M
#define RB_GEMV_MAX_M 16
#endif
#ifndef RB_GEMM_SWAP_MAX_M
#define RB_GEMM_SWAP_MAX_M 256
#endif
static_assert(RB_GEMM_SWAP_MAX_M <= 256, "the swapped kernel's N side holds at most 256 activation rows");

namespace rb {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 128;  // K bytes per stage = one 128-byte swizzle row
constexpr int STAGES = 4;
constexpr int MMA_K = 32;  // int8 K per tcgen05.mma
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 512;
constexpr int NUM_THREADS = 192;
constexpr int EPI_THREADS = 128;
constexpr int BAR_BYTES = 256;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + BAR_BYTES;

// instruction descriptor: D=S32 (bits 4-5 = 2), A/B signed int8 (bits 7-9, 10-12 = 1),
// both K-major, N>>3 at bit 17, M>>4 at bit 24
constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);

struct EpiParams {
  const void* sa;
  const void* sb;
  const void* bias;
  void* out;
  int64_t ldo;
  int64_t M, N, K;
  int sa_dtype, sa_per_row, sb_dtype, bias_dtype, out_dtype;
  int ksplits;         // > 1: each tile covers a K range and writes raw int32 partials
  int32_t* partials;   // [ksplits][M][N] int32 when ksplits > 1
};

// K-major operand tile in shared memory with 128-byte swizzle: rows of 128 B,
// 8-row groups 1024 B apart (SBO), LBO unused (1), version 1, layout 2.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* tm, int c0, int c1, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(IDESC), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

// Operand kinds of the one-SM kernel.  Every kind consumes 32 bytes of K per
// MMA (int8: 32 elements, bf16: 16, fp32 as tf32: 8) and a 128-byte swizzle row
// per stage, so the shared-memory layout and descriptor steps are shared.
enum GemmKind : int { kKindI8 = 0, kKindBF16 = 1, kKindTF32 = 2 };
template <int KIND>
struct KindTraits;
template <>
struct KindTraits<kKindI8> {
  static constexpr int elt = 1;
  static constexpr uint32_t idesc = IDESC;
};
template <>
struct KindTraits<kKindBF16> {  // D = F32 (bits 4-5 = 1), A/B = BF16 (1), K-major
  static constexpr int elt = 2;
  static constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                    ((uint32_t)(BM >> 4) << 24);
};
template <>
struct KindTraits<kKindTF32> {  // D = F32, A/B = TF32 (2), K-major
  static constexpr int elt = 4;
  static constexpr uint32_t idesc = (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                    ((uint32_t)(BM >> 4) << 24);
};

template <int KIND>
__device__ __forceinline__ void umma_kind(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  if constexpr (KIND == kKindI8) {
    umma_i8(d_tmem, adesc, bdesc, acc);
  } else if constexpr (KIND == kKindBF16) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(KindTraits<KIND>::idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
  } else {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(KindTraits<KIND>::idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
  }
}

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 8 consecutive per-column parameters (fp32 or 16-bit) from index i as 4 fp32 pairs
__device__ __forceinline__ void ld_param8(const void* p, int dtype, int64_t i, F2* out) {
  if (dtype == RB_F32) {
    const float4* q = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    const float4 a = __ldg(q), b = __ldg(q + 1);
    out[0] = f2(a.x, a.y); out[1] = f2(a.z, a.w); out[2] = f2(b.x, b.y); out[3] = f2(b.z, b.w);
    return;
  }
  const uint4 w = __ldg(reinterpret_cast<const uint4*>(reinterpret_cast<const uint16_t*>(p) + i));
  const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    if (dtype == RB_BF16) {
      out[k] = f2(bf16_lo(ww[k]), bf16_hi(ww[k]));
    } else {
      const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&ww[k]));
      out[k] = f2(h.x, h.y);
    }
  }
}

// Epilogue for 32 consecutive columns of one row: out = ((f32(acc) * sa) * sb) + bias,
// one rounded fp32 operation at a time (pairs of columns per packed instruction).
// Every array index is static, so the values stay in registers.
// With kF32Acc (the floating-point kinds) the accumulator is fp32 and the
// epilogue is out = acc + bias, without scales.
template <bool kF32Acc = false>
__device__ __forceinline__ void epilogue_32(const uint32_t* r, int64_t row, int64_t col0, float sa_v,
                                            const EpiParams& ep) {
  const int64_t N = ep.N;
  const int ncol = (N - col0 < 32) ? (int)(N - col0) : 32;
  if (ep.out_dtype == RB_I32) {
    int32_t* dst = reinterpret_cast<int32_t*>(ep.out) + row * ep.ldo + col0;
    if (ncol == 32 && aligned(dst, 16)) {
#pragma unroll
      for (int j = 0; j < 32; j += 4)
        *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j < ncol) dst[j] = (int32_t)r[j];
    }
    return;
  }
  F2 v[16];
  if constexpr (kF32Acc) {
#pragma unroll
    for (int j = 0; j < 16; ++j) v[j] = f2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
  } else {
    const F2 sa2 = f2(sa_v, sa_v);
#pragma unroll
    for (int j = 0; j < 16; ++j)
      v[j] = mul2v(f2(__int2float_rn((int)r[2 * j]), __int2float_rn((int)r[2 * j + 1])), sa2);
  }
  const size_t osz = ep.out_dtype == RB_F32 ? 4 : 2;
  const bool vec = ncol == 32 && (kF32Acc || aligned(ep.sb, 16)) && (ep.bias == nullptr || aligned(ep.bias, 16)) &&
                   (col0 & 7) == 0 && ((uintptr_t)ep.out + (row * ep.ldo + col0) * osz) % 32 == 0;
  if (vec) {
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      F2 p[4];
      if constexpr (!kF32Acc) {
        ld_param8(ep.sb, ep.sb_dtype, col0 + 8 * g, p);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[4 * g + k] = mul2v(v[4 * g + k], p[k]);
      }
      if (ep.bias != nullptr) {
        ld_param8(ep.bias, ep.bias_dtype, col0 + 8 * g, p);
#pragma unroll
        for (int k = 0; k < 4; ++k) v[4 * g + k] = add2v(v[4 * g + k], p[k]);
      }
    }
    if (ep.out_dtype == RB_F32) {
      float* dst = reinterpret_cast<float*>(ep.out) + row * ep.ldo + col0;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t w[8];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 x = un(v[4 * g + k]);
          w[2 * k] = __float_as_uint(x.x);
          w[2 * k + 1] = __float_as_uint(x.y);
        }
        stg_v8(dst + 8 * g, w);
      }
    } else {
      uint16_t* dst = reinterpret_cast<uint16_t*>(ep.out) + row * ep.ldo + col0;
      const bool bf = ep.out_dtype == RB_BF16;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint32_t w[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          const float2 x = un(v[8 * h + k]);
          w[k] = bf ? pack_bf16x2(x.x, x.y) : pack_f16x2(x.x, x.y);
        }
        stg_v8(dst + 16 * h, w);
      }
    }
    return;
  }
  // ragged or unaligned columns: element by element
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    if (j >= ncol) break;
    const float2 x2 = un(v[j >> 1]);
    float x = (j & 1) ? x2.y : x2.x;
    if constexpr (!kF32Acc) x = __fmul_rn(x, load_as_f32(ep.sb, ep.sb_dtype, col0 + j));
    if (ep.bias != nullptr) x = __fadd_rn(x, load_as_f32(ep.bias, ep.bias_dtype, col0 + j));
    const int64_t o = row * ep.ldo + col0 + j;
    if (ep.out_dtype == RB_F32) {
      reinterpret_cast<float*>(ep.out)[o] = x;
    } else if (ep.out_dtype == RB_BF16) {
      __nv_bfloat16 hv = __float2bfloat16_rn(x);
      reinterpret_cast<uint16_t*>(ep.out)[o] = *reinterpret_cast<uint16_t*>(&hv);
    } else {
      __half hv = __float2half_rn(x);
      reinterpret_cast<uint16_t*>(ep.out)[o] = *reinterpret_cast<uint16_t*>(&hv);
    }
  }
}

template <int KIND>
__device__ __forceinline__ void gemm_tc_body(const CUtensorMap& tmA, const CUtensorMap& tmB, const EpiParams& ep) {
  constexpr int kElt = KindTraits<KIND>::elt;
  constexpr bool kF32Acc = KIND != kKindI8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;                // [STAGES]  TMA -> MMA
  uint64_t* empty = bars + STAGES;      // [STAGES]  MMA -> TMA
  uint64_t* tfull = bars + 2 * STAGES;  // [2]       MMA -> epilogue
  uint64_t* tempty = tfull + 2;         // [2]       epilogue -> MMA
  uint64_t* done = tempty + 2;          // [1]       MMA drain at exit
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), EPI_THREADS);
    }
    mbar_init(smem_u32(done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int64_t m_tiles = (ep.M + BM - 1) / BM;
  const int64_t n_tiles = (ep.N + BN - 1) / BN;
  const int ksplits = ep.ksplits;
  const int64_t num_tiles = m_tiles * n_tiles * ksplits;
  const int kblocks = (int)((ep.K * kElt + BK - 1) / BK);
  // tile t -> split t % ksplits, n tile (t / ksplits) % n_tiles, m tile t / (ksplits * n_tiles);
  // split s covers k blocks [s*kblocks/ksplits, (s+1)*kblocks/ksplits)
  auto kb_begin = [&](int64_t t) { return (int)((t % ksplits) * kblocks / ksplits); };
  auto kb_end = [&](int64_t t) { return (int)((t % ksplits + 1) * kblocks / ksplits); };
  auto tile_m0 = [&](int64_t t) { return (t / ksplits / n_tiles) * BM; };
  auto tile_n0 = [&](int64_t t) { return ((t / ksplits) % n_tiles) * BN; };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol_a = policy_evict_first(), pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_phase = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        const int m0 = (int)tile_m0(tile);
        const int n0 = (int)tile_n0(tile);
        for (int kb = kb_begin(tile); kb < kb_end(tile); ++kb) {
          if (!mbar_wait_bounded(smem_u32(&empty[stage]), phase ^ 1, kWaitTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb = smem_u32(&full[stage]);
          mbar_arrive_expect_tx(fb, STAGE_BYTES);
          tma_load_2d(smem_u32(sA + stage * A_BYTES), &tmA, kb * (BK / kElt), m0, fb, pol_a);
          tma_load_2d(smem_u32(sB + stage * B_BYTES), &tmB, kb * (BK / kElt), n0, fb, pol_b);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // never leave a bulk copy in flight behind an exiting CTA
      for (int s = 0; s < STAGES; ++s)
        if (issued & (1u << s))
          mbar_wait_bounded(smem_u32(&full[s]), (issued_phase >> s) & 1u, kWaitTimeoutProducer, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // --------------------------------------------------------------- MMA
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int64_t tile = blockIdx.x; tile < num_tiles && ok; tile += gridDim.x) {
        if (!mbar_wait_bounded(smem_u32(&tempty[acc]), acc_phase ^ 1, kWaitTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        const int kb0 = kb_begin(tile);
        for (int kb = kb0; kb < kb_end(tile); ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, kWaitTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_desc(smem_u32(sA + stage * A_BYTES));
          const uint64_t bdesc = sw128_desc(smem_u32(sB + stage * B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / MMA_K; ++k)
            umma_kind<KIND>(d_tmem, adesc + (uint64_t)(k * MMA_K / 16), bdesc + (uint64_t)(k * MMA_K / 16),
                            (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&tfull[acc]));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      // all MMAs issued by this thread are complete once `done` flips
      umma_commit(smem_u32(done));
      mbar_wait_bounded(smem_u32(done), 0, kWaitTimeoutMma, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 are reachable from this warp
    int acc = 0;
    uint32_t acc_phase = 0;
    // split-K tiles store raw int32 partials into their split's slab
    EpiParams pep = ep;
    pep.out_dtype = RB_I32;
    pep.ldo = ep.N;
    for (int64_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x) {
      const int64_t m0 = tile_m0(tile);
      const int64_t n0 = tile_n0(tile);
      if (!mbar_wait_bounded(smem_u32(&tfull[acc]), acc_phase, kWaitTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int64_t row = m0 + quarter * 32 + lane;
      float sa_v = 0.0f;
      if (!kF32Acc && row < ep.M && ep.out_dtype != RB_I32 && ksplits == 1)
        sa_v = load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? row : 0);
      if (ksplits > 1) pep.out = ep.partials + (tile % ksplits) * ep.M * ep.N;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int64_t col0 = n0 + c * 32;
        if (col0 >= ep.N) break;  // warp-uniform
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
        if (row < ep.M) epilogue_32<kF32Acc>(r, row, col0, sa_v, ksplits > 1 ? pep : ep);
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[acc]));
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    w8a8_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ EpiParams ep) {
  gemm_tc_body<kKindI8>(tmA, tmB, ep);
}

// bf16 x bf16 (kind::f16) or fp32 x fp32 (kind::tf32) with fp32 accumulators:
// out = A B^T + bias, the unquantised Linear
template <int KIND>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    fp_gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                      const __grid_constant__ EpiParams ep) {
  gemm_tc_body<KIND>(tmA, tmB, ep);
}

// ----------------------------------------------------------------------------
// Two-SM variant (cta_group::2): a cluster of two CTAs computes a 256x256 tile
// with one tcgen05.mma.cta_group::2 (M=256, N=256, K=32) per K step.  CTA r of
// the pair loads A rows [r*128, r*128+128) and B rows (N) [r*128, r*128+128)
// of the tile into its own shared memory; the MMA, issued by the leader (rank
// 0), reads both CTAs' halves, so each SM's tensor core reads 8 KB of operands
// per 128-clock MMA instead of 12 KB, and TMA writes drop by a third.  Each
// CTA's TMEM holds its own 128 output rows (two 256-column buffers, so the
// epilogue overlaps the next tile).  Loads carry no multicast: every CTA
// fetches its own halves; the leader's full barrier counts both CTAs' bytes.
namespace pair {
constexpr int BM = 256;  // rows per tile (128 per CTA)
constexpr int BK = 128;  // K bytes per stage
constexpr int A_BYTES = 128 * BK;  // this CTA's A half
constexpr int NUM_THREADS = 192;
// Tile width BN = 256 (the default) or 128 (when the 256-wide tiles leave
// pairs idle: at M = 4096, N = 512 there are 32 of them for 74 pairs).  Each
// CTA loads BN / 2 rows of B per stage; the ring takes up to 192 KB.
template <int kBN>
struct Cfg {
  static constexpr int BN = kBN;
  static constexpr int B_BYTES = (kBN / 2) * BK;  // this CTA's B half
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = (192 * 1024) / STAGE_BYTES > 8 ? 8 : (192 * 1024) / STAGE_BYTES;
  static constexpr int TMEM_COLS = 2 * kBN;  // two accumulators
  static constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 + 256;
  static constexpr uint32_t IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                                    ((uint32_t)(BM >> 4) << 24);
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the same shared variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_rank(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* tm, int c0, int c1, uint32_t bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(bar), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void umma_i8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u));
}
// arrive on the barrier at this shared offset in both CTAs of the pair when the MMAs issued so far are done
__device__ __forceinline__ void umma_commit_both(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
      "h"((uint16_t)0x3)
      : "memory");
}
// Arrive on a barrier in a CTA of the cluster.  Used by the epilogue warps to
// hand an accumulator back to the leader's MMA thread: their TMEM reads are
// complete (tcgen05.wait::ld) and ordered before the arrive by
// tcgen05.fence::before_thread_sync, and nothing else they wrote is read by the
// MMA thread, so the default CTA-scope release suffices.  A cluster-scope
// release made each epilogue warp wait for its global stores first (a
// "membar" stall; the SMoE layer at 103k tokens took 0.507 ms with it, 0.480
// ms without).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}

template <int kBN>
__global__ void __launch_bounds__(NUM_THREADS, 1)
    w8a8_gemm_tc_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ EpiParams ep) {
  using C = Cfg<kBN>;
  constexpr int BN = C::BN;
  constexpr int B_BYTES = C::B_BYTES;
  constexpr int STAGE_BYTES = C::STAGE_BYTES;
  constexpr int STAGES = C::STAGES;
  constexpr int TMEM_COLS = C::TMEM_COLS;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* full = bars;                // [STAGES]  leader: TMA bytes of both CTAs -> MMA
  uint64_t* empty = bars + STAGES;      // [STAGES]  both: MMA done with the slot -> TMA
  uint64_t* tfull = bars + 2 * STAGES;  // [2]       both: accumulator ready -> epilogue
  uint64_t* tempty = tfull + 2;         // [2]       leader: both epilogues done -> MMA
  uint64_t* done = tempty + 2;          // [1]       leader: all MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), 2 * 4);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(smem_u32(done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int64_t m_tiles = (ep.M + BM - 1) / BM;
  const int64_t n_tiles = (ep.N + BN - 1) / BN;
  const int ksplits = ep.ksplits;
  // work unit t: K split t % ksplits of output tile t / ksplits (the splits of
  // one tile run on neighbouring pairs); split s covers k blocks
  // [s*kblocks/ksplits, (s+1)*kblocks/ksplits), at least two of them
  const int64_t num_tiles = m_tiles * n_tiles * ksplits;
  const int kblocks = (int)((ep.K + BK - 1) / BK);
  auto kb_begin = [&](int64_t t) { return (int)((t % ksplits) * kblocks / ksplits); };
  auto kb_end = [&](int64_t t) { return (int)((t % ksplits + 1) * kblocks / ksplits); };
  auto tile_mi = [&](int64_t t) { return (t / ksplits) / n_tiles; };
  auto tile_ni = [&](int64_t t) { return (t / ksplits) % n_tiles; };
  const int64_t pair_id = blockIdx.x >> 1;
  const int64_t num_pairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol_a = policy_evict_first(), pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_phase = 0;
      bool ok = true;
      for (int64_t tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        const int m0 = (int)(tile_mi(tile) * BM) + (int)rank * 128;
        const int n0 = (int)(tile_ni(tile) * BN) + (int)rank * (BN / 2);
        const int kb1 = kb_end(tile);
        for (int kb = kb_begin(tile); kb < kb1; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&empty[stage]), phase ^ 1, kWaitTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb_local = smem_u32(&full[stage]);
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * STAGE_BYTES);
          const uint32_t fb = map_rank(fb_local, 0);
          tma_load_2d_pair(smem_u32(sA + stage * A_BYTES), &tmA, kb * BK, m0, fb, pol_a);
          tma_load_2d_pair(smem_u32(sB + stage * B_BYTES), &tmB, kb * BK, n0, fb, pol_b);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (leader) {
        // the leader's full barriers count both CTAs' bytes: drain them before exit
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s))
            mbar_wait_bounded(smem_u32(&full[s]), (issued_phase >> s) & 1u, kWaitTimeoutProducer, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // --------------------------------------------------------------- MMA
      int stage = 0, acc = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int64_t tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        if (!mbar_wait_bounded(smem_u32(&tempty[acc]), acc_phase ^ 1, kWaitTimeoutMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * BN);
        const int kb0 = kb_begin(tile), kb1 = kb_end(tile);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, kWaitTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_desc(smem_u32(sA + stage * A_BYTES));
          const uint64_t bdesc = sw128_desc(smem_u32(sB + stage * B_BYTES));
#pragma unroll
          for (int k = 0; k < BK / MMA_K; ++k)
            umma_i8_pair(d_tmem, adesc + (uint64_t)(k * MMA_K / 16), bdesc + (uint64_t)(k * MMA_K / 16), C::IDESC,
                         (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit_both(smem_u32(&empty[stage]));
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_both(smem_u32(&tfull[acc]));
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1;
      }
      asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(done))
                   : "memory");
      mbar_wait_bounded(smem_u32(done), 0, kWaitTimeoutMma, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const uint32_t tempty_leader0 = map_rank(smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = map_rank(smem_u32(&tempty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    // split-K units store raw int32 partials into their split's [M, N] slab
    EpiParams pep = ep;
    pep.out_dtype = RB_I32;
    pep.ldo = ep.N;
    for (int64_t tile = pair_id; tile < num_tiles; tile += num_pairs) {
      const int64_t m0 = tile_mi(tile) * BM + (int64_t)rank * 128;
      const int64_t n0 = tile_ni(tile) * BN;
      if (!mbar_wait_bounded(smem_u32(&tfull[acc]), acc_phase, kWaitTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int64_t row = m0 + quarter * 32 + lane;
      float sa_v = 0.0f;
      if (row < ep.M && ep.out_dtype != RB_I32 && ksplits == 1)
        sa_v = load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? row : 0);
      if (ksplits > 1) pep.out = ep.partials + (tile % ksplits) * ep.M * ep.N;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int64_t col0 = n0 + c * 32;
        if (col0 >= ep.N) break;  // warp-uniform
        uint32_t r[32];
        tmem_ld32(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN + c * 32), r);
        if (row < ep.M) epilogue_32(r, row, col0, sa_v, ksplits > 1 ? pep : ep);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(acc ? tempty_leader1 : tempty_leader0);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(TMEM_COLS)
                 : "memory");
  }
}

// ----------------------------------------------------------------------------
// K2 with the transformer's first LayerNorm fused (models.py:216-217: layer 0
// starts with residual = x; x = norm1[0](x), x being the RepEncoder output).
// A CTA pair computes 256 x 512 tiles: a whole 512-wide output row sits in one
// CTA's TMEM (two N = 256 MMAs per K step, all 512 columns, one accumulator),
// so the epilogue thread that owns a row writes rep_emb, takes the row's
// LayerNorm statistics in the order of ATen's CUDA LayerNorm for a 512-wide
// row (128 Welford chains of 4 elements, a shuffle-down merge of each group of
// 32 chains, then groups {0,2}, {1,3} and the two halves), and writes
// norm1(rep_emb) from a second read of TMEM.  The main loop waits for the
// epilogue between tiles (one accumulator).  rb_w8a8_gemm_ln uses this kernel
// below M = 4096; from there K2 + ln512_rows_kernel measured faster.
struct LnParams {
  const void* gamma;
  const void* beta;
  int ln_dtype;
  float eps;
  void* out;      // norm1 output [M, 512], same dtype as rep_emb
  int64_t ldo;
};
constexpr int LN_BN = 512;
constexpr int LN_B_BYTES = 2 * 128 * BK;  // this CTA's two 128-row slices of B
constexpr int LN_STAGE_BYTES = A_BYTES + LN_B_BYTES;
constexpr int LN_STAGES = 4;
constexpr int LN_SMEM_BYTES = LN_STAGES * LN_STAGE_BYTES + 1024 + 256;
constexpr uint32_t LN_IDESC = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(256 >> 3) << 17) |
                              ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void welford_push1(float& mean, float& m2, float x, float r) {
  const float delta = __fsub_rn(x, mean);
  mean = __fmaf_rn(delta, r, mean);
  m2 = __fmaf_rn(delta, __fsub_rn(x, mean), m2);
}

// 32 output values of one row (columns col0 .. col0+31) from the int32
// accumulators: ((f32(acc) * sa) * sb) + bias, rounded to the output dtype
// (v[] holds the rounded values widened back to fp32)
__device__ __forceinline__ void ln_out_values(const uint32_t* r, int64_t col0, float sa_v, const EpiParams& ep,
                                              float* v) {
  const F2 sa2 = f2(sa_v, sa_v);
#pragma unroll
  for (int g = 0; g < 4; ++g) {
    F2 sb[4], bi[4];
    ld_param8(ep.sb, ep.sb_dtype, col0 + 8 * g, sb);
    if (ep.bias != nullptr) ld_param8(ep.bias, ep.bias_dtype, col0 + 8 * g, bi);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int j = 8 * g + 2 * k;
      F2 x = mul2v(mul2v(f2(__int2float_rn((int)r[j]), __int2float_rn((int)r[j + 1])), sa2), sb[k]);
      if (ep.bias != nullptr) x = add2v(x, bi[k]);
      float2 xv = un(x);
      if (ep.out_dtype == RB_BF16) {
        xv.x = round_bf16(xv.x);
        xv.y = round_bf16(xv.y);
      } else if (ep.out_dtype == RB_F16) {
        xv.x = __half2float(__float2half_rn(xv.x));
        xv.y = __half2float(__float2half_rn(xv.y));
      }
      v[j] = xv.x;
      v[j + 1] = xv.y;
    }
  }
}

// store 32 fp32 values (already representable in dtype) at dst, 32-byte stores when aligned
__device__ __forceinline__ void ln_store32(void* dst, int dtype, const float* v) {
  if (dtype == RB_F32) {
    float* d = reinterpret_cast<float*>(dst);
    if (aligned(d, 32)) {
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t w[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = __float_as_uint(v[8 * g + k]);
        stg_v8(d + 8 * g, w);
      }
    } else {
#pragma unroll
      for (int k = 0; k < 32; ++k) d[k] = v[k];
    }
    return;
  }
  uint32_t w[16];
#pragma unroll
  for (int k = 0; k < 16; ++k)
    w[k] = dtype == RB_BF16 ? pack_bf16x2(v[2 * k], v[2 * k + 1]) : pack_f16x2(v[2 * k], v[2 * k + 1]);
  uint16_t* d = reinterpret_cast<uint16_t*>(dst);
  if (aligned(d, 32)) {
    stg_v8(d, w);
    stg_v8(d + 16, w + 8);
  } else {
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      d[2 * k] = (uint16_t)(w[k] & 0xffffu);
      d[2 * k + 1] = (uint16_t)(w[k] >> 16);
    }
  }
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    w8a8_gemm_ln_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                             const __grid_constant__ EpiParams ep, const __grid_constant__ LnParams lp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + LN_STAGES * A_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + LN_STAGES * LN_STAGE_BYTES);
  uint64_t* full = bars;                   // [LN_STAGES]  leader: TMA bytes of both CTAs -> MMA
  uint64_t* empty = bars + LN_STAGES;      // [LN_STAGES]  both: MMA done with the slot -> TMA
  uint64_t* tfull = bars + 2 * LN_STAGES;  // [1]          both: accumulator ready -> epilogue
  uint64_t* tempty = tfull + 1;            // [1]          leader: both epilogues done -> MMA
  uint64_t* done = tempty + 1;             // [1]          leader: all MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const bool leader = rank == 0;

  if (threadIdx.x == 0) {
    for (int st = 0; st < LN_STAGES; ++st) {
      mbar_init(smem_u32(&full[st]), 1);
      mbar_init(smem_u32(&empty[st]), 1);
    }
    mbar_init(smem_u32(tfull), 1);
    mbar_init(smem_u32(tempty), 2 * 4);  // one arrival per epilogue warp of both CTAs
    mbar_init(smem_u32(done), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(512)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int64_t num_tiles = (ep.M + BM - 1) / BM;
  const int kblocks = (int)((ep.K + BK - 1) / BK);
  const int64_t pair_id = blockIdx.x >> 1;
  const int64_t num_pairs = gridDim.x >> 1;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol_a = policy_evict_first(), pol_b = policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_phase = 0;
      bool ok = true;
      for (int64_t tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        const int m0 = (int)(tile * BM) + (int)rank * 128;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&empty[stage]), phase ^ 1, kWaitTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb_local = smem_u32(&full[stage]);
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * LN_STAGE_BYTES);
          const uint32_t fb = map_rank(fb_local, 0);
          uint8_t* b = sB + stage * LN_B_BYTES;
          tma_load_2d_pair(smem_u32(sA + stage * A_BYTES), &tmA, kb * BK, m0, fb, pol_a);
          tma_load_2d_pair(smem_u32(b), &tmB, kb * BK, (int)rank * 128, fb, pol_b);
          tma_load_2d_pair(smem_u32(b + 128 * BK), &tmB, kb * BK, 256 + (int)rank * 128, fb, pol_b);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == LN_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (leader) {
        for (int st = 0; st < LN_STAGES; ++st)
          if (issued & (1u << st))
            mbar_wait_bounded(smem_u32(&full[st]), (issued_phase >> st) & 1u, kWaitTimeoutProducer, nullptr);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      // --------------------------------------------------------------- MMA
      int stage = 0;
      uint32_t phase = 0, acc_phase = 0;
      bool ok = true;
      for (int64_t tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        if (!mbar_wait_bounded(smem_u32(tempty), acc_phase ^ 1, kWaitTimeoutMma, abort_flag)) break;
        tc_fence_after();
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, kWaitTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t adesc = sw128_desc(smem_u32(sA + stage * A_BYTES));
          const uint64_t bdesc0 = sw128_desc(smem_u32(sB + stage * LN_B_BYTES));
          const uint64_t bdesc1 = sw128_desc(smem_u32(sB + stage * LN_B_BYTES + 128 * BK));
#pragma unroll
          for (int k = 0; k < BK / MMA_K; ++k) {
            const uint32_t accf = (kb > 0 || k > 0) ? 1u : 0u;
            umma_i8_pair(tmem_base, adesc + (uint64_t)(k * MMA_K / 16), bdesc0 + (uint64_t)(k * MMA_K / 16),
                         LN_IDESC, accf);
            umma_i8_pair(tmem_base + 256, adesc + (uint64_t)(k * MMA_K / 16), bdesc1 + (uint64_t)(k * MMA_K / 16),
                         LN_IDESC, accf);
          }
          umma_commit_both(smem_u32(&empty[stage]));
          if (++stage == LN_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_both(smem_u32(tfull));
        acc_phase ^= 1;
      }
      asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                       smem_u32(done))
                   : "memory");
      mbar_wait_bounded(smem_u32(done), 0, kWaitTimeoutMma, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const uint32_t tempty_leader = map_rank(smem_u32(tempty), 0);
    const uint32_t lane_base = tmem_base + ((uint32_t)(quarter * 32) << 16);
    uint32_t acc_phase = 0;
    const bool bf_ln = lp.ln_dtype == RB_BF16;
    for (int64_t tile = pair_id; tile < num_tiles; tile += num_pairs) {
      if (!mbar_wait_bounded(smem_u32(tfull), acc_phase, kWaitTimeoutEpilogue, abort_flag)) break;
      tc_fence_after();
      const int64_t row = tile * BM + (int64_t)rank * 128 + quarter * 32 + lane;
      const bool live = row < ep.M;
      const float sa_v = live ? load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? row : 0) : 0.0f;
      uint8_t* out_row = reinterpret_cast<uint8_t*>(ep.out) + (live ? row : 0) * ep.ldo * dtype_size(ep.out_dtype);
      // pass 1: rep_emb, and per 128-column group (an ATen warp of 32 chains of
      // 4 columns) the merged Welford state
      float gmean[4], gm2[4];
#pragma unroll 1
      for (int w = 0; w < 4; ++w) {
        float cm[32], cq[32];  // chains 32w .. 32w+31 (columns 128w + 4j .. +3)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t r[32];
          float v[32];
          tmem_ld32(lane_base + (uint32_t)(128 * w + 32 * c), r);
          ln_out_values(r, 128 * w + 32 * c, sa_v, ep, v);
          if (live) ln_store32(out_row + (int64_t)(128 * w + 32 * c) * dtype_size(ep.out_dtype), ep.out_dtype, v);
#pragma unroll
          for (int q = 0; q < 8; q += 2) {  // chains 8c + q, 8c + q + 1: columns 4q .. 4q+7 of this chunk
            Welford2 st{f2(0.0f, 0.0f), f2(0.0f, 0.0f)};
            welford_push2(st, f2(v[4 * q], v[4 * q + 4]), 1.0f);
            welford_push2(st, f2(v[4 * q + 1], v[4 * q + 5]), 0.5f);
            welford_push2(st, f2(v[4 * q + 2], v[4 * q + 6]), 1.0f / 3.0f);
            welford_push2(st, f2(v[4 * q + 3], v[4 * q + 7]), 0.25f);
            const float2 m = un(st.mean), q2 = un(st.m2);
            cm[8 * c + q] = m.x;
            cm[8 * c + q + 1] = m.y;
            cq[8 * c + q] = q2.x;
            cq[8 * c + q + 1] = q2.y;
          }
        }
        // shuffle-down merge of the 32 chains: chain j takes chain j + d
        float cnt = 4.0f;
#pragma unroll
        for (int d = 16; d >= 1; d >>= 1) {
#pragma unroll
          for (int j = 0; j < d; ++j) {
            const float2 mq = welford_merge1(cm[j], cq[j], cm[j + d], cq[j + d], cnt);
            cm[j] = mq.x;
            cq[j] = mq.y;
          }
          cnt = __fadd_rn(cnt, cnt);
        }
        gmean[w] = cm[0];
        gm2[w] = cq[0];
      }
      // the accumulator is no longer needed: let the MMA warp start the next tile
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(tempty_leader);
      // groups 0, 1 take groups 2, 3 (128 elements each), then 0 takes 1 (256 each)
      const float2 g02 = welford_merge1(gmean[0], gm2[0], gmean[2], gm2[2], 128.0f);
      const float2 g13 = welford_merge1(gmean[1], gm2[1], gmean[3], gm2[3], 128.0f);
      const float2 fin = welford_merge1(g02.x, g02.y, g13.x, g13.y, 256.0f);
      const float mean = fin.x;
      const float rstd = rsqrtf(__fadd_rn(__fdiv_rn(fin.y, 512.0f), lp.eps));
      // pass 2: norm1(rep_emb) = fma(gamma, rstd * (x - mean), beta), rounded to the
      // dtype, from the row this thread stored in pass 1 (program order makes it visible)
      uint8_t* ln_row = reinterpret_cast<uint8_t*>(lp.out) + (live ? row : 0) * lp.ldo * dtype_size(ep.out_dtype);
      if (live) {
#pragma unroll 1
        for (int c = 0; c < LN_BN / 32; ++c) {
          float v[32];
          const uint8_t* src = out_row + (int64_t)(32 * c) * dtype_size(ep.out_dtype);
          if (ep.out_dtype == RB_F32) {
            const float4* q = reinterpret_cast<const float4*>(src);
#pragma unroll
            for (int k = 0; k < 8; ++k) {
              const float4 t = q[k];
              v[4 * k] = t.x; v[4 * k + 1] = t.y; v[4 * k + 2] = t.z; v[4 * k + 3] = t.w;
            }
          } else {
            const uint4* q = reinterpret_cast<const uint4*>(src);
            const bool bf = ep.out_dtype == RB_BF16;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint4 t = q[k];
              const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                if (bf) {
                  v[8 * k + 2 * h] = bf16_lo(w[h]);
                  v[8 * k + 2 * h + 1] = bf16_hi(w[h]);
                } else {
                  const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[h]));
                  v[8 * k + 2 * h] = f.x;
                  v[8 * k + 2 * h + 1] = f.y;
                }
              }
            }
          }
#pragma unroll
          for (int gq = 0; gq < 4; ++gq) {
            F2 gg[4], bb[4];
            ld_param8(lp.gamma, lp.ln_dtype, 32 * c + 8 * gq, gg);
            ld_param8(lp.beta, lp.ln_dtype, 32 * c + 8 * gq, bb);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const float2 g2 = un(gg[k]), b2 = un(bb[k]);
              const int j = 8 * gq + 2 * k;
              v[j] = __fmaf_rn(g2.x, __fmul_rn(rstd, __fsub_rn(v[j], mean)), b2.x);
              v[j + 1] = __fmaf_rn(g2.y, __fmul_rn(rstd, __fsub_rn(v[j + 1], mean)), b2.y);
            }
          }
#pragma unroll
          for (int k = 0; k < 32; ++k) {
            if (ep.out_dtype == RB_BF16) v[k] = round_bf16(v[k]);
            else if (ep.out_dtype == RB_F16) v[k] = __half2float(__float2half_rn(v[k]));
          }
          ln_store32(ln_row + (int64_t)(32 * c) * dtype_size(ep.out_dtype), ep.out_dtype, v);
        }
      }
      (void)bf_ln;
      acc_phase ^= 1;
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(512) : "memory");
  }
}
}  // namespace pair

// out[m, n] = epilogue(acc) for one element (the finalize and small-M paths)
__device__ __forceinline__ void epilogue_one(int32_t acc, int64_t m, int64_t n, const EpiParams& ep) {
  if (ep.out_dtype == RB_I32) {
    reinterpret_cast<int32_t*>(ep.out)[m * ep.ldo + n] = acc;
    return;
  }
  float v = __int2float_rn(acc);
  v = __fmul_rn(v, load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? m : 0));
  v = __fmul_rn(v, load_as_f32(ep.sb, ep.sb_dtype, n));
  if (ep.bias != nullptr) v = __fadd_rn(v, load_as_f32(ep.bias, ep.bias_dtype, n));
  if (ep.out_dtype == RB_F32) {
    reinterpret_cast<float*>(ep.out)[m * ep.ldo + n] = v;
  } else if (ep.out_dtype == RB_BF16) {
    reinterpret_cast<__nv_bfloat16*>(ep.out)[m * ep.ldo + n] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(ep.out)[m * ep.ldo + n] = __float2half_rn(v);
  }
}

// Split-K reduction: out[m, n] = epilogue(sum over the splits of the int32
// partials).  int32 addition is exact (modulo 2^32, in any order), so the
// result equals the unsplit GEMM's bit for bit.  A thread owns 4 consecutive
// columns of one row: one 16-byte load per split (four splits in flight), the
// scales and bias as 4-wide vectors and one store; the epilogue's fp32 steps
// are the GEMM kernels' ((acc * sa) * sb) + bias, one rounded op at a time.
// Ragged or unaligned groups go element by element.
constexpr int kFinCols = 4;

__device__ __forceinline__ void ld_param4(const void* p, int dtype, int64_t i, float* out) {
  if (dtype == RB_F32) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i));
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    return;
  }
  const uint2 w = __ldg(reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + i));
  if (dtype == RB_BF16) {
    out[0] = bf16_lo(w.x); out[1] = bf16_hi(w.x); out[2] = bf16_lo(w.y); out[3] = bf16_hi(w.y);
  } else {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
    out[0] = a.x; out[1] = a.y; out[2] = b.x; out[3] = b.y;
  }
}

__global__ void __launch_bounds__(256) splitk_finalize_kernel(const __grid_constant__ EpiParams ep) {
  const uint64_t groups = (uint64_t)((ep.N + kFinCols - 1) / kFinCols);  // column groups per row
  const uint64_t total = (uint64_t)ep.M * groups;
  const int64_t slab = ep.M * ep.N;
  const size_t osz = ep.out_dtype == RB_F32 || ep.out_dtype == RB_I32 ? 4 : 2;
  const bool vec_in = ep.N % 4 == 0 && aligned(ep.partials, 16);
  const bool vec_par = ep.out_dtype == RB_I32 ||
                       (aligned(ep.sb, 16) && (ep.bias == nullptr || aligned(ep.bias, 16)));
  const bool vec_out = aligned(ep.out, 16) && (ep.ldo * (int64_t)osz) % 16 == 0;
  for (uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x; t < total;
       t += (uint64_t)gridDim.x * blockDim.x) {
    const int64_t m = (int64_t)(t / groups);
    const int64_t n0 = (int64_t)(t % groups) * kFinCols;
    if (!(vec_in && vec_par && vec_out && n0 + kFinCols <= ep.N)) {
      for (int j = 0; j < kFinCols && n0 + j < ep.N; ++j) {
        int32_t acc = 0;
        for (int s = 0; s < ep.ksplits; ++s) acc += ep.partials[s * slab + m * ep.N + n0 + j];
        epilogue_one(acc, m, n0 + j, ep);
      }
      continue;
    }
    uint32_t a[4] = {0u, 0u, 0u, 0u};
    const uint4* src = reinterpret_cast<const uint4*>(ep.partials + m * ep.N + n0);
#pragma unroll 4
    for (int s = 0; s < ep.ksplits; ++s) {
      const uint4 x = __ldcs(src + s * (slab / 4));
      a[0] += x.x; a[1] += x.y; a[2] += x.z; a[3] += x.w;
    }
    if (ep.out_dtype == RB_I32) {
      *reinterpret_cast<uint4*>(reinterpret_cast<int32_t*>(ep.out) + m * ep.ldo + n0) = make_uint4(a[0], a[1], a[2], a[3]);
      continue;
    }
    const float sa_v = load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? m : 0);
    float sb[4], bi[4];
    ld_param4(ep.sb, ep.sb_dtype, n0, sb);
    if (ep.bias != nullptr) ld_param4(ep.bias, ep.bias_dtype, n0, bi);
    float v[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      v[k] = __fmul_rn(__fmul_rn(__int2float_rn((int)a[k]), sa_v), sb[k]);
      if (ep.bias != nullptr) v[k] = __fadd_rn(v[k], bi[k]);
    }
    if (ep.out_dtype == RB_F32) {
      *reinterpret_cast<float4*>(reinterpret_cast<float*>(ep.out) + m * ep.ldo + n0) = make_float4(v[0], v[1], v[2], v[3]);
    } else {
      const bool bf = ep.out_dtype == RB_BF16;
      const uint32_t w0 = bf ? pack_bf16x2(v[0], v[1]) : pack_f16x2(v[0], v[1]);
      const uint32_t w1 = bf ? pack_bf16x2(v[2], v[3]) : pack_f16x2(v[2], v[3]);
      *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(ep.out) + m * ep.ldo + n0) = make_uint2(w0, w1);
    }
  }
}

// Small M (M <= kGemvMaxM): reading the [N, K] weight once is the whole cost
// (7.3 MB for the RepEncoder's linear), and a tensor-core tile would be 1/8
// full.  One launch, no workspace.  A cluster of kGvSplit CTAs owns kGvCols
// output columns; CTA r of the cluster covers the r-th 1/kGvSplit of K.  Warp w
// owns columns 4(w%4)..4(w%4)+3 of the cluster (for 9-16 rows, warps 4-7 take
// rows 8-15 of the same columns) and lane l the 16-byte K chunks l, l+32,
// l+64, l+96 of each round of 128 chunks: a thread issues all sixteen of its
// weight loads before the first product, so the whole weight is in flight at
// once (the grid is resident in one wave), and the round's A slice (M x 2 KB)
// comes into shared memory with cp.async.  Products are exact dp4a; the warp's
// rows x 4 sums are reduce-scattered over its lanes, written
// into the leader CTA's shared memory through the cluster's distributed shared
// memory, and summed there in CTA order before the usual epilogue.  int32
// addition (modulo 2^32, like the tensor core's) is associative, so the result
// equals the tiled kernels' bit for bit.
constexpr int kGemvMaxM = 16;
constexpr int kGvSplit = 8;     // CTAs per cluster, along K
constexpr int kGvCols = 16;     // output columns per cluster
constexpr int kGvThreads = 128; // 4 warps x 4 columns per group of rows
// rows of A per group of 4 warps: 16 rows run as two groups of 8, so that a
// thread carries 32 sums instead of 64 and twice the warps share an SM (the
// M = 16 case is latency-bound on its dp4a chains at 167 registers per thread)
__host__ __device__ constexpr int gv_groups(int mt) { return mt >= 16 ? 2 : 1; }
constexpr int kGvIt = 4;        // chunks per lane per round
constexpr int kGvRound = 32 * kGvIt;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

template <int MT>
__global__ void __launch_bounds__(kGvThreads * gv_groups(MT), gv_groups(MT) > 1 ? 2 : 3)
    w8a8_gemv_kernel(const int8_t* __restrict__ A, int64_t lda, const int8_t* __restrict__ B, int64_t ldb,
                     const __grid_constant__ EpiParams ep) {
  constexpr int kGroups = gv_groups(MT);
  constexpr int RG = MT / kGroups;              // rows per group
  constexpr int kThreads = kGvThreads * kGroups;
  constexpr int V = RG * 4;                     // sums per warp: its group's rows x 4 columns
  __shared__ __align__(16) int4 sA[MT][kGvRound];
  __shared__ __align__(16) uint32_t red[kGvSplit][4 * kGroups][V];
  // every CTA of the cluster has started before any writes into the leader's
  // shared memory (the matching wait comes after the products)
  asm volatile("barrier.cluster.arrive.relaxed;" ::: "memory");
  const uint32_t rank = pair::cluster_rank();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int cw = warp & 3;       // the warp's 4 columns: 4*cw .. 4*cw+3 of the cluster's 16
  const int row0 = (warp >> 2) * RG;  // the warp's rows: row0 .. row0+RG-1
  const int64_t n0 = (int64_t)(blockIdx.x / kGvSplit) * kGvCols;
  const int M = (int)ep.M;
  const int64_t chunks = ep.K / 16;
  const int64_t per_cta = (chunks + kGvSplit - 1) / kGvSplit;
  const int64_t k0 = (int64_t)rank * per_cta;
  const int64_t k_end = min(chunks, k0 + per_cta);
  // Programmatic dependent launch: the next kernel on the stream may start now
  // (a kernel launched that way waits for this grid to complete before it
  // reads what this grid writes).  While the previous kernel finishes, this
  // CTA requests its weight slice into L2, then waits until that kernel's
  // writes are visible before it reads anything.  A prefetch has no
  // architectural effect: a weight written by the previous kernel is still
  // read fresh from L2 after the wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (k_end > k0) {
    const int64_t seg = (k_end - k0) * 16;  // bytes of one weight row in this CTA's K range
    const int lines = (int)((seg + 127) / 128);
    for (int i = threadIdx.x; i < kGvCols * lines; i += kThreads) {
      const int64_t n = n0 + i / lines;
      const int64_t off = min((int64_t)(i % lines) * 128, seg - 1);
      if (n < ep.N) asm volatile("prefetch.global.L2 [%0];" ::"l"(B + n * ldb + k0 * 16 + off));
    }
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // the leader's epilogue operands, requested now so that their latency
  // overlaps the loads and products instead of following the last barrier
  constexpr int kPer = (MT * kGvCols + kThreads - 1) / kThreads;
  float e_sa[kPer], e_sb[kPer], e_bi[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    e_sa[j] = e_sb[j] = e_bi[j] = 0.0f;
    const int o = threadIdx.x + j * kThreads;
    const int m = o / kGvCols;
    const int64_t n = n0 + o % kGvCols;
    if (rank == 0 && ep.out_dtype != RB_I32 && o < MT * kGvCols && m < M && n < ep.N) {
      e_sa[j] = load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? m : 0);
      e_sb[j] = load_as_f32(ep.sb, ep.sb_dtype, n);
      if (ep.bias != nullptr) e_bi[j] = load_as_f32(ep.bias, ep.bias_dtype, n);
    }
  }
  int32_t acc[RG][4];
#pragma unroll
  for (int m = 0; m < RG; ++m)
#pragma unroll
    for (int c = 0; c < 4; ++c) acc[m][c] = 0;
  for (int64_t r0 = k0; r0 < k_end; r0 += kGvRound) {
    // A rows of this round into shared memory (zeros past M or the slice)
    for (int i = threadIdx.x; i < MT * kGvRound; i += kThreads) {
      const int m = i / kGvRound, q = i % kGvRound;
      const bool ok = m < M && r0 + q < k_end;
      cp_async16((uint32_t)__cvta_generic_to_shared(&sA[m][q]), ok ? A + m * lda + (r0 + q) * 16 : A, ok ? 16u : 0u);
    }
    // every weight load of the round before the first product
    int4 b[kGvIt][4];
#pragma unroll
    for (int it = 0; it < kGvIt; ++it) {
      const int64_t q = r0 + lane + 32 * it;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int64_t n = n0 + 4 * cw + c;
        b[it][c] = (q < k_end && n < ep.N) ? __ldg(reinterpret_cast<const int4*>(B + n * ldb) + q)
                                           : make_int4(0, 0, 0, 0);
      }
    }
    cp_async_wait_all();
    __syncthreads();
#pragma unroll
    for (int it = 0; it < kGvIt; ++it) {
#pragma unroll
      for (int m = 0; m < RG; ++m) {
        const int4 a = sA[row0 + m][lane + 32 * it];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          int v = acc[m][c];
          v = __dp4a(a.x, b[it][c].x, v);
          v = __dp4a(a.y, b[it][c].y, v);
          v = __dp4a(a.z, b[it][c].z, v);
          v = __dp4a(a.w, b[it][c].w, v);
          acc[m][c] = v;
        }
      }
    }
    __syncthreads();  // sA is rewritten by the next round
  }
  // reduce-scatter over the warp: each xor step halves the values a lane
  // carries until one is left (two when V = 64), then plain xor sums.  Value
  // j = 4m + c ends on lane j << (5 - log2 V) (and its xor partners) for
  // V <= 32, and on lane j / 2 for V = 64.
  uint32_t v[V];
#pragma unroll
  for (int m = 0; m < RG; ++m)
#pragma unroll
    for (int c = 0; c < 4; ++c) v[4 * m + c] = (uint32_t)acc[m][c];
  int h = V;
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    if (h > 2 || (h == 2 && V <= 32)) {
      h >>= 1;
      const bool upper = (lane & d) != 0;
#pragma unroll
      for (int i = 0; i < V / 2; ++i) {
        if (i < h) {
          const uint32_t send = upper ? v[i] : v[i + h];
          const uint32_t keep = upper ? v[i + h] : v[i];
          v[i] = keep + __shfl_xor_sync(0xffffffffu, send, d);
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < 2; ++i)
        if (i < h) v[i] += __shfl_xor_sync(0xffffffffu, v[i], d);
    }
  }
  asm volatile("barrier.cluster.wait;" ::: "memory");
  const uint32_t red_local = (uint32_t)__cvta_generic_to_shared(&red[rank][warp][0]);
  const uint32_t red_leader = pair::map_rank(red_local, 0);
  if constexpr (V == 64) {
    asm volatile("st.shared::cluster.v2.u32 [%0], {%1, %2};" ::"r"(red_leader + 8u * lane), "r"(v[0]), "r"(v[1])
                 : "memory");
  } else {
    constexpr int kShift = 5 - (V == 4 ? 2 : V == 8 ? 3 : V == 16 ? 4 : 5);
    if ((lane & ((1 << kShift) - 1)) == 0)
      asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(red_leader + 4u * (lane >> kShift)), "r"(v[0])
                   : "memory");
  }
  pair::cluster_sync_all();
  if (rank != 0) return;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int o = threadIdx.x + j * kThreads;
    const int m = o / kGvCols, col = o % kGvCols;
    const int64_t n = n0 + col;
    if (o < MT * kGvCols && m < M && n < ep.N) {
      uint32_t sum = 0;
#pragma unroll
      for (int r = 0; r < kGvSplit; ++r) sum += red[r][(m / RG) * 4 + (col >> 2)][4 * (m % RG) + (col & 3)];
      if (ep.out_dtype == RB_I32) {
        reinterpret_cast<int32_t*>(ep.out)[m * ep.ldo + n] = (int32_t)sum;
        continue;
      }
      // the epilogue_one arithmetic on the preloaded operands
      float v = __fmul_rn(__fmul_rn(__int2float_rn((int32_t)sum), e_sa[j]), e_sb[j]);
      if (ep.bias != nullptr) v = __fadd_rn(v, e_bi[j]);
      if (ep.out_dtype == RB_F32) {
        reinterpret_cast<float*>(ep.out)[m * ep.ldo + n] = v;
      } else if (ep.out_dtype == RB_BF16) {
        reinterpret_cast<__nv_bfloat16*>(ep.out)[m * ep.ldo + n] = __float2bfloat16_rn(v);
      } else {
        reinterpret_cast<__half*>(ep.out)[m * ep.ldo + n] = __float2half_rn(v);
      }
    }
  }
}

// ----------------------------------------------------------------------------
// Small M (1 <= M <= kSwapMaxM): the operands swapped and K split over a
// cluster.  Out^T = W * A^T: the weight's 128-row tile is the MMA's M side
// and the activation rows (padded to MP, a multiple of 16) its N side, so
// one tcgen05.mma.kind::i8 (M = 128, N = MP, K = 32) covers every row of A.
// A cluster of kSwapSplit CTAs owns 128 output columns; CTA r takes the r-th
// share of the K blocks.  Each CTA accumulates its int32 partial in TMEM,
// stages it in shared memory ([128 columns][MP rows], padded against bank
// conflicts), and after a cluster barrier CTA r sums the 8 columns
// [8r, 8r + 8) across the cluster's shared memories (distributed shared
// memory, int32 addition: exact in any order), runs the epilogue on them and
// writes each output row's 8 values with one 16-byte store.
// One launch, no workspace; the weight streams through all clusters' SMs at
// once.  No TMA load carries a multicast.
namespace swp {
constexpr int kSplit = 16;         // CTAs per cluster, along K (non-portable cluster size)
constexpr int BK = 128;            // K bytes per stage
constexpr int kMaxStages = 16;
constexpr int kMaxMP = 256;
constexpr int W_BYTES = 128 * BK;  // weight rows of the tile
constexpr int NUM_THREADS = 192;
constexpr int kColsPerCta = 128 / kSplit;  // output columns each CTA reduces (8)
// shared memory: a ring of stages of 16 KB of weight + MP x 128 B of A (as many
// as fit, so that for small M every K block of the CTA is requested at once),
// reused for the partial [128][MP + 4] int32 after the main loop
constexpr int kRing = 192 * 1024;
// after the barriers: the epilogue's per-row activation scales (kMaxMP) and the
// CTA's 8 columns' weight scales and bias, loaded while the main loop runs
constexpr int kEpiBytes = (kMaxMP + 2 * 8) * 4;
constexpr int kBarBytes = 512;  // full/empty[kMaxStages], tfull, TMEM address, abort flag (272 B)
constexpr int SMEM_BYTES = kRing + 1024 + kBarBytes + kEpiBytes;

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void umma_i8_n(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}

__device__ __forceinline__ uint4 ld_cluster_v4(uint32_t cluster_addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(cluster_addr)
               : "memory");
  return v;
}

// one output element: ((f32(acc) * sa) * sb) + bias in the output dtype, or the raw int32
__device__ __forceinline__ void store_one(const EpiParams& ep, int64_t m, int64_t n, int32_t acc) {
  const int64_t o = m * ep.ldo + n;
  if (ep.out_dtype == RB_I32) {
    reinterpret_cast<int32_t*>(ep.out)[o] = acc;
    return;
  }
  float v = __fmul_rn(__int2float_rn(acc), load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? m : 0));
  v = __fmul_rn(v, load_as_f32(ep.sb, ep.sb_dtype, n));
  if (ep.bias != nullptr) v = __fadd_rn(v, load_as_f32(ep.bias, ep.bias_dtype, n));
  if (ep.out_dtype == RB_F32) {
    reinterpret_cast<float*>(ep.out)[o] = v;
  } else if (ep.out_dtype == RB_BF16) {
    reinterpret_cast<__nv_bfloat16*>(ep.out)[o] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(ep.out)[o] = __float2half_rn(v);
  }
}

// one output element's bits: the raw int32, or ((f32(acc) * sa) * sb) + bias
// rounded to the output dtype (in the low bits for 16-bit dtypes)
__device__ __forceinline__ int32_t out_bits(const EpiParams& ep, float sa, float sb, float bias, int64_t n,
                                            int32_t acc) {
  if (ep.out_dtype == RB_I32 || n >= ep.N) return acc;
  float v = __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sb);
  if (ep.bias != nullptr) v = __fadd_rn(v, bias);
  if (ep.out_dtype == RB_F32) return __float_as_int(v);
  if (ep.out_dtype == RB_BF16) return (int32_t)__bfloat16_as_ushort(__float2bfloat16_rn(v));
  return (int32_t)__half_as_ushort(__float2half_rn(v));
}

// the 8 staged outputs of row m, columns n0 .. n0+7 (n0 a multiple of 8): one
// or two 16-byte stores when the row is whole and aligned, else one by one
__device__ __forceinline__ void store_row8(const EpiParams& ep, int64_t m, int64_t n0, const int32_t* bits) {
  const int esz = dtype_size(ep.out_dtype);
  const int64_t o = m * ep.ldo + n0;
  char* base = reinterpret_cast<char*>(ep.out) + o * esz;
  const uint4 b0 = *reinterpret_cast<const uint4*>(bits), b1 = *reinterpret_cast<const uint4*>(bits + 4);
  const bool vec = n0 + 8 <= ep.N && (reinterpret_cast<uintptr_t>(base) & 15) == 0;
  if (esz == 4) {
    if (vec) {
      reinterpret_cast<uint4*>(base)[0] = b0;
      reinterpret_cast<uint4*>(base)[1] = b1;
    } else {
      for (int j = 0; j < 8 && n0 + j < ep.N; ++j) reinterpret_cast<int32_t*>(base)[j] = bits[j];
    }
    return;
  }
  if (vec) {
    *reinterpret_cast<uint4*>(base) = make_uint4((b0.x & 0xffffu) | (b0.y << 16), (b0.z & 0xffffu) | (b0.w << 16),
                                                 (b1.x & 0xffffu) | (b1.y << 16), (b1.z & 0xffffu) | (b1.w << 16));
  } else {
    for (int j = 0; j < 8 && n0 + j < ep.N; ++j) reinterpret_cast<uint16_t*>(base)[j] = (uint16_t)bits[j];
  }
}

// tmW: the weight [N, K] (128-row boxes); tmA: the activations [M, K] (MP-row boxes)
__global__ void __launch_bounds__(NUM_THREADS, 1)
    w8a8_gemm_swap_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmA,
                          const __grid_constant__ EpiParams ep, int mp) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  const int a_bytes = mp * BK;
  const int stage_bytes = W_BYTES + a_bytes;                // 1024-aligned: mp is a multiple of 16
  const int kStages = min(kMaxStages, kRing / stage_bytes);  // 4 at mp = 256, 10 at mp = 16
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kRing);
  uint64_t* full = bars;                // [kMaxStages]  TMA -> MMA
  uint64_t* empty = bars + kMaxStages;  // [kMaxStages]  MMA -> TMA
  uint64_t* tfull = empty + kMaxStages; // [1]           MMA -> epilogue
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tfull + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* s_sa = reinterpret_cast<float*>(smem + kRing + kBarBytes);  // [mp] activation scale per row
  float* s_sb = s_sa + kMaxMP;                                 // [8] weight scales of the CTA's columns
  float* s_bias = s_sb + 8;                                    // [8] bias of the CTA's columns (0 without)
  int32_t* part = reinterpret_cast<int32_t*>(smem);  // after the main loop: [128][mp + 4]
  const int ldp = mp + 4;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = pair::cluster_rank();
  const int64_t n_tile0 = (int64_t)(blockIdx.x / kSplit) * 128;
  const int kblocks = (int)((ep.K + BK - 1) / BK);
  const int kb0 = (int)((int64_t)rank * kblocks / kSplit);
  const int kb1 = (int)((int64_t)(rank + 1) * kblocks / kSplit);
  const bool has_k = kb1 > kb0;
  const uint32_t tmem_cols = mp <= 32 ? 32u : (mp <= 64 ? 64u : (mp <= 128 ? 128u : 256u));
  const uint32_t idesc = (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(mp >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);

  if (threadIdx.x == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(smem_u32(&full[st]), 1);
      mbar_init(smem_u32(&empty[st]), 1);
    }
    mbar_init(smem_u32(tfull), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  // Programmatic dependent launch (as in w8a8_gemv_kernel): the next kernel
  // may start; while the previous kernel finishes, this CTA requests its
  // weight boxes into L2 (a prefetch has no architectural effect) and sets up
  // its barriers and TMEM; every read of data follows griddepcontrol.wait.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    for (int kb = kb0; kb < kb1; ++kb)
      asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                       reinterpret_cast<uint64_t>(&tmW)),
                   "r"(kb * BK), "r"((int)n_tile0)
                   : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(tmem_cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    if (lane == 0 && has_k) {
      // ---------------------------------------------------------- producer
      const uint64_t pol = policy_evict_first();
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_phase = 0;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&empty[stage]), phase ^ 1, kWaitTimeoutProducer, abort_flag)) break;
        const uint32_t fb = smem_u32(&full[stage]);
        uint8_t* sW = smem + stage * stage_bytes;
        mbar_arrive_expect_tx(fb, (uint32_t)stage_bytes);
        tma_load_2d(smem_u32(sW), &tmW, kb * BK, (int)n_tile0, fb, pol);
        tma_load_2d(smem_u32(sW + W_BYTES), &tmA, kb * BK, 0, fb, pol);
        issued |= 1u << stage;
        issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      // never leave a bulk copy in flight behind an exiting CTA (or a reused ring)
      for (int st = 0; st < kStages; ++st)
        if (issued & (1u << st))
          mbar_wait_bounded(smem_u32(&full[st]), (issued_phase >> st) & 1u, kWaitTimeoutProducer, nullptr);
    }
  } else if (warp == 1) {
    if (lane == 0 && has_k) {
      // --------------------------------------------------------------- MMA
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, kWaitTimeoutMma, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint8_t* sW = smem + stage * stage_bytes;
        const uint64_t wdesc = sw128_desc(smem_u32(sW));
        const uint64_t adesc = sw128_desc(smem_u32(sW + W_BYTES));
#pragma unroll
        for (int k = 0; k < BK / MMA_K; ++k)
          umma_i8_n(tmem_base, wdesc + (uint64_t)(k * MMA_K / 16), adesc + (uint64_t)(k * MMA_K / 16), idesc,
                    (kb > kb0 || k > 0) ? 1u : 0u);
        umma_commit(smem_u32(&empty[stage]));
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1;
        }
      }
      // the partial is complete (and the ring idle) once tfull flips
      umma_commit(smem_u32(tfull));
      if (!ok) *abort_flag = 1;
    }
  } else {
    // ------------- epilogue operands into shared memory while the main loop runs
    if (ep.out_dtype != RB_I32) {
      const int et = threadIdx.x - 64;  // 0 .. 127
      for (int m = et; m < (int)ep.M; m += 128) s_sa[m] = load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? m : 0);
      if (et < 8) {
        const int64_t n = n_tile0 + (int64_t)rank * kColsPerCta + et;
        s_sb[et] = n < ep.N ? load_as_f32(ep.sb, ep.sb_dtype, n) : 0.0f;
        s_bias[et] = (ep.bias != nullptr && n < ep.N) ? load_as_f32(ep.bias, ep.bias_dtype, n) : 0.0f;
      }
    }
    // --------------------------------------- TMEM -> shared partial [128][ldp]
    const int quarter = warp & 3;
    const int row = quarter * 32 + lane;  // TMEM lane = output column of the tile
    bool ready = !has_k;
    if (has_k) ready = mbar_wait_bounded(smem_u32(tfull), 0, kWaitTimeoutEpilogue, abort_flag) && !*abort_flag;
    tc_fence_after();
    int32_t* dst = part + row * ldp;
    for (int c = 0; c < mp; c += 16) {
      uint32_t r[16];
      if (has_k && ready) {
        tmem_ld16(tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)c, r);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) r[i] = 0u;  // no K share (or a failed wait): a zero partial
      }
#pragma unroll
      for (int i = 0; i < 16; i += 4)
        *reinterpret_cast<uint4*>(dst + c + i) = make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]);
    }
  }
  tc_fence_before();
  __syncthreads();
  pair::cluster_sync_all();  // every CTA's partial is in its shared memory

  // ---- CTA `rank` sums columns [8 rank, 8 rank + 8) of the tile over the
  // cluster (consecutive threads read consecutive rows of a column: each
  // warp's remote reads are contiguous), applies the epilogue and stages the
  // [M][8] outputs in its own shared memory, then writes one row's 8 outputs
  // per thread (one 16-byte store for bf16 / f16)
  int32_t* stage_out = part + 128 * ldp;  // [mp][8] raw output bits (int32 or the output dtype's)
  const int64_t n0 = n_tile0 + (int64_t)rank * kColsPerCta;
  {
    const int m4n = (int)((ep.M + 3) / 4);     // groups of 4 rows of A that exist
    const int items = kColsPerCta * m4n;       // (column, 4 consecutive rows of A)
    const uint32_t part_addr = smem_u32(part);
    for (int it = threadIdx.x; it < items; it += NUM_THREADS) {
      const int j = it / m4n;
      const int m4 = (it % m4n) * 4;
      const int col = (int)rank * kColsPerCta + j;
      const uint32_t off = (uint32_t)((col * ldp + m4) * 4);
      uint4 v[kSplit];
#pragma unroll
      for (int q = 0; q < kSplit; ++q) v[q] = ld_cluster_v4(pair::map_rank(part_addr + off, (uint32_t)q));
      uint4 acc = v[0];
#pragma unroll
      for (int q = 1; q < kSplit; ++q) {
        acc.x += v[q].x;
        acc.y += v[q].y;
        acc.z += v[q].z;
        acc.w += v[q].w;
      }
      const uint32_t a4[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        stage_out[(m4 + i) * kColsPerCta + j] = out_bits(ep, s_sa[m4 + i < ep.M ? m4 + i : 0], s_sb[j], s_bias[j],
                                                         n0 + j, (int32_t)a4[i]);
    }
  }
  __syncthreads();
  for (int m = threadIdx.x; m < (int)ep.M; m += NUM_THREADS) store_row8(ep, m, n0, stage_out + m * kColsPerCta);
  pair::cluster_sync_all();  // no CTA leaves while another still reads its partial
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(tmem_cols)
                 : "memory");
  }
}
}  // namespace swp

// CUDA-core GEMM for shapes the tensor-map path cannot take (K % 16 != 0,
// unaligned operands, K == 0).  One thread per output element.
__global__ void w8a8_gemm_simple_kernel(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb,
                                        const __grid_constant__ EpiParams ep) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= ep.M * ep.N) return;
  const int64_t m = idx / ep.N, n = idx % ep.N;
  int32_t acc = 0;
  const int8_t* a = A + m * lda;
  const int8_t* b = B + n * ldb;
  for (int64_t k = 0; k < ep.K; ++k) acc += (int32_t)a[k] * (int32_t)b[k];
  if (ep.out_dtype == RB_I32) {
    reinterpret_cast<int32_t*>(ep.out)[m * ep.ldo + n] = acc;
    return;
  }
  float v = __int2float_rn(acc);
  v = __fmul_rn(v, load_as_f32(ep.sa, ep.sa_dtype, ep.sa_per_row ? m : 0));
  v = __fmul_rn(v, load_as_f32(ep.sb, ep.sb_dtype, n));
  if (ep.bias != nullptr) v = __fadd_rn(v, load_as_f32(ep.bias, ep.bias_dtype, n));
  if (ep.out_dtype == RB_F32) {
    reinterpret_cast<float*>(ep.out)[m * ep.ldo + n] = v;
  } else if (ep.out_dtype == RB_BF16) {
    reinterpret_cast<__nv_bfloat16*>(ep.out)[m * ep.ldo + n] = __float2bfloat16_rn(v);
  } else {
    reinterpret_cast<__half*>(ep.out)[m * ep.ldo + n] = __float2half_rn(v);
  }
}

// CUDA-core fp GEMM for shapes the tensor-map path cannot take: fp32 sum of
// products in K order, then + bias.  One thread per output element.
template <typename T>
__global__ void fp_gemm_simple_kernel(const T* A, int64_t lda, const T* B, int64_t ldb,
                                      const __grid_constant__ EpiParams ep) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= ep.M * ep.N) return;
  const int64_t m = idx / ep.N, n = idx % ep.N;
  float acc = 0.0f;
  for (int64_t k = 0; k < ep.K; ++k) acc = __fmaf_rn((float)A[m * lda + k], (float)B[n * ldb + k], acc);
  if (ep.bias != nullptr) acc = __fadd_rn(acc, load_as_f32(ep.bias, ep.bias_dtype, n));
  const int64_t o = m * ep.ldo + n;
  if (ep.out_dtype == RB_F32) {
    reinterpret_cast<float*>(ep.out)[o] = acc;
  } else if (ep.out_dtype == RB_BF16) {
    reinterpret_cast<__nv_bfloat16*>(ep.out)[o] = __float2bfloat16_rn(acc);
  } else {
    reinterpret_cast<__half*>(ep.out)[o] = __float2half_rn(acc);
  }
}

// --------------------------------------------------------------------- host
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode;
}

// 2-D tensor map of a row-major [outer, inner] matrix (inner and box_inner in
// elements of `dt`, ld_bytes the row pitch in bytes), 128-byte swizzle
static int make_tmap(CUtensorMap* tm, const void* base, int64_t inner, int64_t outer, int64_t ld_bytes,
                     uint32_t box_inner, uint32_t box_outer, CUtensorMapDataType dt = CU_TENSOR_MAP_DATA_TYPE_UINT8) {
  auto enc = encode_fn();
  if (enc == nullptr) return fail(RB_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
  cuuint64_t strides[1] = {(cuuint64_t)ld_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(tm, dt, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(RB_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return RB_OK;
}

static std::once_flag g_attr_once[64];
static std::once_flag g_pair_attr_once[64];
static std::once_flag g_fp_attr_once[64];
static std::once_flag g_swap_attr_once[64];
static std::once_flag g_ln_attr_once[64];

}  // namespace tc
}  // namespace rb

using namespace rb;

// the split-K reduction over M x ceil(N / 4) column groups, one per thread
static int launch_splitk_finalize(const rb::tc::EpiParams& ep, cudaStream_t st) {
  const int64_t groups = ep.M * ((ep.N + rb::tc::kFinCols - 1) / rb::tc::kFinCols);
  const int64_t blocks = std::min<int64_t>((groups + 255) / 256, (int64_t)sm_count() * 16);
  rb::tc::splitk_finalize_kernel<<<(unsigned)blocks, 256, 0, st>>>(ep);
  return check_cuda(cudaGetLastError(), "splitk_finalize_kernel launch");
}

// split-K factor for the one-SM kernel (1 = no split): enough (m, n, k) tiles to
// cover the SMs, at least two K blocks per split, and at most kMaxKSplits: every
// split writes and the finalize reads back an M x N int32 partial, which past
// 16 splits costs more than the extra SMs gain (K = 14336, N = 512 on a B200:
// 17.6 -> 15.0 us at M = 256, 12.5 -> 11.8 us at M = 64, M = 17 unchanged).
constexpr int64_t kMaxKSplits = 16;
static int choose_ksplits(int64_t M, int64_t N, int64_t K) {
  using namespace rb::tc;
  if (M >= RB_GEMM_PAIR_MIN_M || M <= tc::kGemvMaxM || M <= RB_GEMV_MAX_M || M <= RB_GEMM_SWAP_MAX_M || K <= 0 ||
      K % 16 != 0)
    return 1;
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int64_t kblocks = (K + BK - 1) / BK;
  int64_t s = std::min<int64_t>(sm_count() / std::max<int64_t>(tiles, 1), kblocks / 2);
  return (int)std::max<int64_t>(1, std::min<int64_t>(s, kMaxKSplits));
}

// split-K factor for the two-SM kernel: when the 256 x 256 tiles cover at most
// half of the CTA pairs, each tile's K range is split over pairs (int32
// partials summed by splitk_finalize_kernel).  Then ksplits * M * N <=
// pairs * 256 * 256 int32, the same bound as the one-SM kernel's split.
static int choose_pair_ksplits(int64_t M, int64_t N, int64_t K) {
  using namespace rb::tc;
  if (M < RB_GEMM_PAIR_SPLIT_MIN_M || K <= 0 || K % 16 != 0) return 1;
  const int64_t pairs = sm_count() / 2;
  const int64_t t256 = ((M + 255) / 256) * ((N + 255) / 256);
  const int64_t kblocks = (K + pair::BK - 1) / pair::BK;
  if (2 * t256 > pairs) return 1;
  const int64_t s = std::min<int64_t>(std::min<int64_t>(pairs / t256, kblocks / 2), kMaxKSplits);
  return (int)std::max<int64_t>(1, s);
}

extern "C" int64_t rb_w8a8_gemm_workspace_size(int64_t M, int64_t N, int64_t K) {
  if (M <= 0 || N <= 0) return 0;
  const int pks = choose_pair_ksplits(M, N, K);
  const int s = (M >= RB_GEMM_PAIR_MIN_M || pks > 1) ? pks : choose_ksplits(M, N, K);
  return s > 1 ? (int64_t)s * M * N : 0;
}

extern "C" int rb_w8a8_gemm_ws(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int64_t M, int64_t N,
                               int64_t K, const void* sa, int sa_dtype, int sa_per_row, const void* sb, int sb_dtype,
                               const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
                               int32_t* workspace, int64_t workspace_elems, void* stream) {
  using namespace rb::tc;
  if (M < 0 || N < 0 || K < 0) return fail(RB_ERR_VALUE, "negative GEMM shape");
  if (M == 0 || N == 0) return RB_OK;
  if (A == nullptr || B == nullptr || out == nullptr) return fail(RB_ERR_VALUE, "null operand");
  if (lda < K || ldb < K || ldo < N) return fail(RB_ERR_VALUE, "leading dimension smaller than the row");
  if (out_dtype != RB_BF16 && out_dtype != RB_F16 && out_dtype != RB_F32 && out_dtype != RB_I32)
    return fail(RB_ERR_VALUE, "out dtype must be bf16/f16/f32/i32");
  if (out_dtype != RB_I32) {
    if (sa == nullptr || sb == nullptr) return fail(RB_ERR_VALUE, "scales must be given");
    auto fdt = [](int d) { return d == RB_F32 || d == RB_BF16 || d == RB_F16; };
    if (!fdt(sa_dtype) || !fdt(sb_dtype) || (bias != nullptr && !fdt(bias_dtype)))
      return fail(RB_ERR_VALUE, "scale/bias dtypes must be f32/bf16/f16");
  }
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL) return fail(RB_ERR_UNSUPPORTED, "dimension above 2^31-1");
  EpiParams ep;
  ep.sa = sa;
  ep.sb = sb;
  ep.bias = bias;
  ep.out = out;
  ep.ldo = ldo;
  ep.M = M;
  ep.N = N;
  ep.K = K;
  ep.sa_dtype = sa_dtype;
  ep.sa_per_row = sa_per_row;
  ep.sb_dtype = sb_dtype;
  ep.bias_dtype = bias_dtype;
  ep.out_dtype = out_dtype;
  ep.ksplits = 1;
  ep.partials = nullptr;
  cudaStream_t st = (cudaStream_t)stream;

  const bool tma_ok = K > 0 && K % 16 == 0 && lda % 16 == 0 && ldb % 16 == 0 && aligned(A, 16) &&
                      aligned(B, 16) && device_is_sm100();
  if (!tma_ok) {
    if (!device_is_sm100()) return fail(RB_ERR_DEVICE, "rb_w8a8_gemm needs an sm_100 (B200) device");
    const int64_t total = M * N;
    const int threads = 256;
    w8a8_gemm_simple_kernel<<<(unsigned)((total + threads - 1) / threads), threads, 0, st>>>(A, lda, B, ldb, ep);
    return check_cuda(cudaGetLastError(), "w8a8_gemm_simple_kernel launch");
  }
  if (M <= RB_GEMV_MAX_M && M <= kGemvMaxM) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((N + kGvCols - 1) / kGvCols) * kGvSplit));
    cfg.blockDim = dim3(kGvThreads * (M > 8 ? gv_groups(16) : 1));
    cfg.dynamicSmemBytes = 0;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = kGvSplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // may start before the previous kernel on the stream completes (the
    // kernel's griddepcontrol.wait orders every read after that kernel)
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    cudaError_t le;
    if (M <= 1) le = cudaLaunchKernelEx(&cfg, w8a8_gemv_kernel<1>, A, lda, B, ldb, ep);
    else if (M <= 2) le = cudaLaunchKernelEx(&cfg, w8a8_gemv_kernel<2>, A, lda, B, ldb, ep);
    else if (M <= 4) le = cudaLaunchKernelEx(&cfg, w8a8_gemv_kernel<4>, A, lda, B, ldb, ep);
    else if (M <= 8) le = cudaLaunchKernelEx(&cfg, w8a8_gemv_kernel<8>, A, lda, B, ldb, ep);
    else le = cudaLaunchKernelEx(&cfg, w8a8_gemv_kernel<16>, A, lda, B, ldb, ep);
    if (le != cudaSuccess) return check_cuda(le, "w8a8_gemv_kernel launch");
    return check_cuda(cudaGetLastError(), "w8a8_gemv_kernel launch");
  }
  int dev = 0;
  cudaGetDevice(&dev);
  int rc;
  if (M <= RB_GEMM_SWAP_MAX_M) {
    // swapped operands, K split over a 16-CTA cluster, partials summed over DSMEM
    const int mp = (int)((M + 15) / 16 * 16);
    CUtensorMap tmW, tmAct;
    rc = make_tmap(&tmW, B, K, N, ldb, swp::BK, 128);
    if (rc) return rc;
    rc = make_tmap(&tmAct, A, K, M, lda, swp::BK, (uint32_t)mp);
    if (rc) return rc;
    cudaError_t se = cudaSuccess;
    std::call_once(g_swap_attr_once[dev & 63], [&] {
      se = cudaFuncSetAttribute(swp::w8a8_gemm_swap_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                swp::SMEM_BYTES);
      if (se == cudaSuccess)
        se = cudaFuncSetAttribute(swp::w8a8_gemm_swap_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    });
    if (se != cudaSuccess) return check_cuda(se, "cudaFuncSetAttribute(w8a8_gemm_swap_kernel)");
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)(((N + 127) / 128) * swp::kSplit));
    cfg.blockDim = dim3(swp::NUM_THREADS);
    cfg.dynamicSmemBytes = swp::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = swp::kSplit;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // see w8a8_gemv_kernel
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return check_cuda(cudaLaunchKernelEx(&cfg, swp::w8a8_gemm_swap_kernel, tmW, tmAct, ep, mp),
                      "w8a8_gemm_swap_kernel launch");
  }
  // the two-SM kernel split along K (needs the workspace) from M = RB_GEMM_PAIR_SPLIT_MIN_M
  int pks = choose_pair_ksplits(M, N, K);
  if (pks > 1 && (workspace == nullptr || workspace_elems < (int64_t)pks * M * N)) pks = 1;
  if (M >= RB_GEMM_PAIR_MIN_M || pks > 1) {
    // two-SM tiles: each CTA of a pair loads 128 rows of A and BN/2 of B.  A
    // 128-wide tile re-reads A twice as often and runs about 1.45x longer per
    // output column than a 256-wide one (L2-bound: K = 14336, N = 512 on a
    // B200), so the narrow tiles are used only when they save whole waves:
    // M = 4096 takes 50.4 us with them, 57.4 us without; M = 32768 246 against 169
    const int pairs_avail = sm_count() / 2;
    const int64_t mt = (M + pair::BM - 1) / pair::BM;
    const int64_t t256 = mt * ((N + 255) / 256), t128 = mt * ((N + 127) / 128);
    const int64_t cost256 = 4 * ((t256 + pairs_avail - 1) / pairs_avail);  // in quarter-units of a 128-wide tile
    const int64_t cost128 = 3 * ((t128 + pairs_avail - 1) / pairs_avail);
    // too few tiles for half the pairs: 256-wide tiles split along K instead
    if (pks > 1) {
      ep.ksplits = pks;
      ep.partials = workspace;
    }
    const bool narrow = pks == 1 && cost128 < cost256;
    const int bn = narrow ? 128 : 256;
    CUtensorMap tpA, tpB;
    rc = make_tmap(&tpA, A, K, M, lda, pair::BK, 128);
    if (rc) return rc;
    rc = make_tmap(&tpB, B, K, N, ldb, pair::BK, (uint32_t)(bn / 2));
    if (rc) return rc;
    cudaError_t pe = cudaSuccess;
    std::call_once(g_pair_attr_once[dev & 63], [&] {
      pe = cudaFuncSetAttribute(pair::w8a8_gemm_tc_pair_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                pair::Cfg<256>::SMEM_BYTES);
      if (pe == cudaSuccess)
        pe = cudaFuncSetAttribute(pair::w8a8_gemm_tc_pair_kernel<128>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                  pair::Cfg<128>::SMEM_BYTES);
    });
    if (pe != cudaSuccess) return check_cuda(pe, "cudaFuncSetAttribute(w8a8_gemm_tc_pair_kernel)");
    const int64_t ptiles = (narrow ? t128 : t256) * pks;
    const int pairs = (int)std::min<int64_t>(ptiles, pairs_avail);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * pairs);
    cfg.blockDim = dim3(pair::NUM_THREADS);
    cfg.dynamicSmemBytes = narrow ? pair::Cfg<128>::SMEM_BYTES : pair::Cfg<256>::SMEM_BYTES;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (narrow)
      return check_cuda(cudaLaunchKernelEx(&cfg, pair::w8a8_gemm_tc_pair_kernel<128>, tpA, tpB, ep),
                        "w8a8_gemm_tc_pair_kernel<128> launch");
    rc = check_cuda(cudaLaunchKernelEx(&cfg, pair::w8a8_gemm_tc_pair_kernel<256>, tpA, tpB, ep),
                    "w8a8_gemm_tc_pair_kernel<256> launch");
    if (rc || pks == 1) return rc;
    return launch_splitk_finalize(ep, st);
  }
  // one-SM tiles, split along K when the (m, n) tiles alone cannot fill the GPU
  int ks = choose_ksplits(M, N, K);
  if (ks > 1) {
    if (workspace == nullptr || workspace_elems < (int64_t)ks * M * N) {
      ks = 1;  // no (or too small a) workspace: run unsplit
    } else {
      ep.ksplits = ks;
      ep.partials = workspace;
    }
  }
  CUtensorMap tmA, tmB;
  rc = make_tmap(&tmA, A, K, M, lda, BK, BM);
  if (rc) return rc;
  rc = make_tmap(&tmB, B, K, N, ldb, BK, BN);
  if (rc) return rc;
  cudaError_t attr_err = cudaSuccess;
  std::call_once(g_attr_once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(w8a8_gemm_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return check_cuda(attr_err, "cudaFuncSetAttribute(w8a8_gemm_tc_kernel)");
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * ep.ksplits;
  const int grid = (int)std::min<int64_t>(tiles, sm_count());
  w8a8_gemm_tc_kernel<<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tmA, tmB, ep);
  rc = check_cuda(cudaGetLastError(), "w8a8_gemm_tc_kernel launch");
  if (rc || ep.ksplits == 1) return rc;
  return launch_splitk_finalize(ep, st);
}

extern "C" int rb_w8a8_gemm(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int64_t M, int64_t N,
                            int64_t K, const void* sa, int sa_dtype, int sa_per_row, const void* sb, int sb_dtype,
                            const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
                            void* stream) {
  return rb_w8a8_gemm_ws(A, lda, B, ldb, M, N, K, sa, sa_dtype, sa_per_row, sb, sb_dtype, bias, bias_dtype, out,
                         ldo, out_dtype, nullptr, 0, stream);
}

// ----------------------------------------------------------------------------
// K2 + the transformer's layer-0 LayerNorm(512): out as rb_w8a8_gemm, and
// ln_out = LayerNorm(out) with gamma/beta (ATen's CUDA order, bit for bit).
// ----------------------------------------------------------------------------
// LayerNorm over rows of 512 in the order of ATen's CUDA LayerNorm for a
// 512-wide row (128 threads, thread c a Welford chain over columns
// 4c .. 4c+3; shuffle-down merge of each warp's 32 chains; warps {0,1} take
// {2,3}, then warp 0 takes warp 1; rstd = rsqrtf(m2 / 512 + eps)), one warp per
// row: lane l carries chains l, l + 32, l + 64, l + 96 (lane l of ATen's four
// warps) as two packed pairs.  Used after K2 for the encoder's norm1 when the
// separate pass is faster than the fused epilogue.
namespace ln512 {
constexpr int kRowsPerCta = 8;

__device__ __forceinline__ void ld4(const void* p, int dtype, int64_t i, float* v) {
  if (dtype == RB_F32) {
    const float4 t = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(p) + i);
    v[0] = t.x; v[1] = t.y; v[2] = t.z; v[3] = t.w;
  } else {
    const uint2 t = *reinterpret_cast<const uint2*>(reinterpret_cast<const uint16_t*>(p) + i);
    if (dtype == RB_BF16) {
      v[0] = bf16_lo(t.x); v[1] = bf16_hi(t.x); v[2] = bf16_lo(t.y); v[3] = bf16_hi(t.y);
    } else {
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&t.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&t.y));
      v[0] = a.x; v[1] = a.y; v[2] = b.x; v[3] = b.y;
    }
  }
}

__device__ __forceinline__ void st4(void* p, int dtype, int64_t i, const float* v) {
  if (dtype == RB_F32) {
    *reinterpret_cast<float4*>(reinterpret_cast<float*>(p) + i) = make_float4(v[0], v[1], v[2], v[3]);
  } else if (dtype == RB_BF16) {
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + i) =
        make_uint2(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]));
  } else {
    *reinterpret_cast<uint2*>(reinterpret_cast<uint16_t*>(p) + i) =
        make_uint2(pack_f16x2(v[0], v[1]), pack_f16x2(v[2], v[3]));
  }
}

__global__ void __launch_bounds__(32 * kRowsPerCta)
    ln512_rows_kernel(const void* x, int64_t ldx, int x_dtype, const void* gamma, const void* beta, int ln_dtype,
                      float eps, void* y, int64_t ldy, int64_t M) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * kRowsPerCta + (threadIdx.x >> 5);
  if (row >= M) return;
  float v[4][4];  // [q][e]: column 4 (32 q + lane) + e, chain 32 q + lane
#pragma unroll
  for (int q = 0; q < 4; ++q) ld4(x, x_dtype, row * ldx + 4 * (32 * q + lane), v[q]);
  Welford2 a{f2(0.0f, 0.0f), f2(0.0f, 0.0f)}, b = a;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float rc = 1.0f / (float)(e + 1);  // cuWelfordOnlineSum's 1 / (count + 1)
    welford_push2(a, f2(v[0][e], v[2][e]), rc);
    welford_push2(b, f2(v[1][e], v[3][e]), rc);
  }
  float cnt = 4.0f;
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) {
    Welford2 oa, ob;
    oa.mean.r = __shfl_down_sync(0xffffffffu, a.mean.r, d);
    oa.m2.r = __shfl_down_sync(0xffffffffu, a.m2.r, d);
    ob.mean.r = __shfl_down_sync(0xffffffffu, b.mean.r, d);
    ob.m2.r = __shfl_down_sync(0xffffffffu, b.m2.r, d);
    a = welford_merge2(a, oa, cnt);
    b = welford_merge2(b, ob, cnt);
    cnt = __fadd_rn(cnt, cnt);
  }
  float mean = 0.0f, rstd = 0.0f;
  if (lane == 0) {
    const float2 am = un(a.mean), aq = un(a.m2), bm = un(b.mean), bq = un(b.m2);
    const float2 w02 = welford_merge1(am.x, aq.x, am.y, aq.y, cnt);  // cnt = 128
    const float2 w13 = welford_merge1(bm.x, bq.x, bm.y, bq.y, cnt);
    const float2 fin = welford_merge1(w02.x, w02.y, w13.x, w13.y, 256.0f);
    mean = fin.x;
    rstd = rsqrtf(__fadd_rn(__fdiv_rn(fin.y, 512.0f), eps));
  }
  mean = __shfl_sync(0xffffffffu, mean, 0);
  rstd = __shfl_sync(0xffffffffu, rstd, 0);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    const int64_t c = 4 * (32 * q + lane);
    float g[4], bb[4], o[4];
    ld4(gamma, ln_dtype, c, g);
    ld4(beta, ln_dtype, c, bb);
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = __fmaf_rn(g[e], __fmul_rn(rstd, __fsub_rn(v[q][e], mean)), bb[e]);
    st4(y, x_dtype, row * ldy + c, o);
  }
}
}  // namespace ln512

extern "C" int rb_w8a8_gemm_ln(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int64_t M, int64_t N,
                               int64_t K, const void* sa, int sa_dtype, int sa_per_row, const void* sb, int sb_dtype,
                               const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
                               const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps, void* ln_out,
                               int64_t ldl, void* stream) {
  using namespace rb::tc;
  if (M < 0 || K < 0) return fail(RB_ERR_VALUE, "negative GEMM shape");
  if (N != pair::LN_BN) return fail(RB_ERR_UNSUPPORTED, "rb_w8a8_gemm_ln needs N == 512, got %lld", (long long)N);
  if (M == 0) return RB_OK;
  if (A == nullptr || B == nullptr || out == nullptr || ln_out == nullptr) return fail(RB_ERR_VALUE, "null operand");
  if (lda < K || ldb < K || ldo < N || ldl < N) return fail(RB_ERR_VALUE, "leading dimension smaller than the row");
  if (out_dtype != RB_BF16 && out_dtype != RB_F16 && out_dtype != RB_F32)
    return fail(RB_ERR_VALUE, "out dtype must be bf16/f16/f32");
  auto fdt = [](int d) { return d == RB_F32 || d == RB_BF16 || d == RB_F16; };
  if (sa == nullptr || sb == nullptr || !fdt(sa_dtype) || !fdt(sb_dtype) || (bias != nullptr && !fdt(bias_dtype)))
    return fail(RB_ERR_VALUE, "scales (and bias) must be given as f32/bf16/f16");
  if (!aligned(sb, 16) || (bias != nullptr && !aligned(bias, 16)))
    return fail(RB_ERR_VALUE, "per-channel scales and bias must be 16-byte aligned");
  if (ln_gamma == nullptr || ln_beta == nullptr || !fdt(ln_dtype))
    return fail(RB_ERR_VALUE, "LayerNorm gamma/beta must be given as f32/bf16/f16");
  if (!aligned(ln_gamma, 16) || !aligned(ln_beta, 16)) return fail(RB_ERR_VALUE, "gamma/beta must be 16-byte aligned");
  if (!aligned(out, 16) || (ldo * dtype_size(out_dtype)) % 16 != 0)
    return fail(RB_ERR_VALUE, "out rows must be 16-byte aligned");
  if (M > 0x7fffffffLL || K > 0x7fffffffLL) return fail(RB_ERR_UNSUPPORTED, "dimension above 2^31-1");
  if (!device_is_sm100()) return fail(RB_ERR_DEVICE, "rb_w8a8_gemm_ln needs an sm_100 (B200) device");
  if (!(K > 0 && K % 16 == 0 && lda % 16 == 0 && ldb % 16 == 0 && aligned(A, 16) && aligned(B, 16)))
    return fail(RB_ERR_UNSUPPORTED, "rb_w8a8_gemm_ln needs K %% 16 == 0 and 16-byte aligned operand rows");
  // From M = 4096 (the CTA-pair GEMM, no workspace) K2 followed by a separate
  // LayerNorm(512) pass over its output, still in L2, is faster than the fused
  // epilogue (0.62 against 0.70 ms at M = 103k on a B200: the 512-column tiles
  // of the fused kernel fill fewer waves and its tensor pipe idles while the
  // epilogue runs); both give the same bits.
  if (M >= RB_GEMM_PAIR_MIN_M && aligned(ln_out, 16) && (ldl * dtype_size(out_dtype)) % 16 == 0) {
    int rc2 = rb_w8a8_gemm_ws(A, lda, B, ldb, M, N, K, sa, sa_dtype, sa_per_row, sb, sb_dtype, bias, bias_dtype, out,
                              ldo, out_dtype, nullptr, 0, stream);
    if (rc2) return rc2;
    const unsigned blocks = (unsigned)((M + ln512::kRowsPerCta - 1) / ln512::kRowsPerCta);
    ln512::ln512_rows_kernel<<<blocks, 32 * ln512::kRowsPerCta, 0, (cudaStream_t)stream>>>(
        out, ldo, out_dtype, ln_gamma, ln_beta, ln_dtype, eps, ln_out, ldl, M);
    return check_cuda(cudaGetLastError(), "ln512_rows_kernel launch");
  }
  EpiParams ep{};
  ep.sa = sa;
  ep.sb = sb;
  ep.bias = bias;
  ep.out = out;
  ep.ldo = ldo;
  ep.M = M;
  ep.N = N;
  ep.K = K;
  ep.sa_dtype = sa_dtype;
  ep.sa_per_row = sa_per_row;
  ep.sb_dtype = sb_dtype;
  ep.bias_dtype = bias_dtype;
  ep.out_dtype = out_dtype;
  ep.ksplits = 1;
  pair::LnParams lp{};
  lp.gamma = ln_gamma;
  lp.beta = ln_beta;
  lp.ln_dtype = ln_dtype;
  lp.eps = eps;
  lp.out = ln_out;
  lp.ldo = ldl;
  CUtensorMap tpA, tpB;
  int rc = make_tmap(&tpA, A, K, M, lda, pair::BK, 128);
  if (rc) return rc;
  rc = make_tmap(&tpB, B, K, N, ldb, pair::BK, 128);
  if (rc) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t pe = cudaSuccess;
  std::call_once(g_ln_attr_once[dev & 63], [&] {
    pe = cudaFuncSetAttribute(pair::w8a8_gemm_ln_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              pair::LN_SMEM_BYTES);
  });
  if (pe != cudaSuccess) return check_cuda(pe, "cudaFuncSetAttribute(w8a8_gemm_ln_pair_kernel)");
  const int64_t tiles = (M + pair::BM - 1) / pair::BM;
  const int pairs = (int)std::min<int64_t>(tiles, sm_count() / 2);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * pairs);
  cfg.blockDim = dim3(pair::NUM_THREADS);
  cfg.dynamicSmemBytes = pair::LN_SMEM_BYTES;
  cfg.stream = (cudaStream_t)stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return check_cuda(cudaLaunchKernelEx(&cfg, pair::w8a8_gemm_ln_pair_kernel, tpA, tpB, ep, lp),
                    "w8a8_gemm_ln_pair_kernel launch");
}

// ----------------------------------------------------------------------------
// Unquantised Linear on the tensor cores: out = A B^T + bias with A [M, K] and
// B [N, K] both bf16 (tcgen05 kind::f16) or both fp32 (kind::tf32: operands
// rounded to tf32 by the tensor core, products accumulated in fp32), fp32
// accumulators in TMEM, bias added in fp32, out in bf16 / fp16 / fp32.
extern "C" int rb_fp_gemm(const void* A, int ab_dtype, int64_t lda, const void* B, int64_t ldb, int64_t M, int64_t N,
                          int64_t K, const void* bias, int bias_dtype, void* out, int64_t ldo, int out_dtype,
                          void* stream) {
  using namespace rb::tc;
  if (M < 0 || N < 0 || K < 0) return fail(RB_ERR_VALUE, "negative GEMM shape");
  if (M == 0 || N == 0) return RB_OK;
  if (ab_dtype != RB_BF16 && ab_dtype != RB_F32) return fail(RB_ERR_VALUE, "rb_fp_gemm operands must be bf16 or f32");
  if (A == nullptr || B == nullptr || out == nullptr) return fail(RB_ERR_VALUE, "null operand");
  if (lda < K || ldb < K || ldo < N) return fail(RB_ERR_VALUE, "leading dimension smaller than the row");
  if (out_dtype != RB_BF16 && out_dtype != RB_F16 && out_dtype != RB_F32)
    return fail(RB_ERR_VALUE, "out dtype must be bf16/f16/f32");
  if (bias != nullptr && bias_dtype != RB_F32 && bias_dtype != RB_BF16 && bias_dtype != RB_F16)
    return fail(RB_ERR_VALUE, "bias dtype must be f32/bf16/f16");
  if (M > 0x7fffffffLL || N > 0x7fffffffLL || K > 0x7fffffffLL) return fail(RB_ERR_UNSUPPORTED, "dimension above 2^31-1");
  if (!device_is_sm100()) return fail(RB_ERR_DEVICE, "rb_fp_gemm needs an sm_100 (B200) device");
  EpiParams ep{};
  ep.bias = bias;
  ep.out = out;
  ep.ldo = ldo;
  ep.M = M;
  ep.N = N;
  ep.K = K;
  ep.bias_dtype = bias_dtype;
  ep.out_dtype = out_dtype;
  ep.ksplits = 1;
  cudaStream_t st = (cudaStream_t)stream;
  const int elt = ab_dtype == RB_BF16 ? 2 : 4;
  // TMA needs 16-byte aligned bases and row pitches; K > 0
  const bool tma_ok = K > 0 && (K * elt) % 16 == 0 && (lda * elt) % 16 == 0 && (ldb * elt) % 16 == 0 &&
                      aligned(A, 16) && aligned(B, 16);
  if (!tma_ok) {
    const int64_t total = M * N;
    const unsigned blocks = (unsigned)((total + 255) / 256);
    if (ab_dtype == RB_BF16)
      fp_gemm_simple_kernel<__nv_bfloat16><<<blocks, 256, 0, st>>>(
          static_cast<const __nv_bfloat16*>(A), lda, static_cast<const __nv_bfloat16*>(B), ldb, ep);
    else
      fp_gemm_simple_kernel<float><<<blocks, 256, 0, st>>>(static_cast<const float*>(A), lda,
                                                           static_cast<const float*>(B), ldb, ep);
    return check_cuda(cudaGetLastError(), "fp_gemm_simple_kernel launch");
  }
  const CUtensorMapDataType dt = ab_dtype == RB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
  CUtensorMap tmA, tmB;
  int rc = make_tmap(&tmA, A, K, M, lda * elt, BK / elt, BM, dt);
  if (rc) return rc;
  rc = make_tmap(&tmB, B, K, N, ldb * elt, BK / elt, BN, dt);
  if (rc) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(g_fp_attr_once[dev & 63], [&] {
    attr_err = cudaFuncSetAttribute(fp_gemm_tc_kernel<kKindBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    SMEM_BYTES);
    if (attr_err == cudaSuccess)
      attr_err = cudaFuncSetAttribute(fp_gemm_tc_kernel<kKindTF32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return check_cuda(attr_err, "cudaFuncSetAttribute(fp_gemm_tc_kernel)");
  const int64_t tiles = ((M + BM - 1) / BM) * ((N + BN - 1) / BN);
  const int grid = (int)std::min<int64_t>(tiles, sm_count());
  if (ab_dtype == RB_BF16)
    fp_gemm_tc_kernel<kKindBF16><<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tmA, tmB, ep);
  else
    fp_gemm_tc_kernel<kKindTF32><<<grid, NUM_THREADS, SMEM_BYTES, st>>>(tmA, tmB, ep);
  return check_cuda(cudaGetLastError(), "fp_gemm_tc_kernel launch");
}

// ----------------------------------------------------------------------------
// Allocation-free entry point.  Some callers cannot allocate device memory on
// their own: embedders whose device memory belongs to another allocator (a
// framework's caching pool, a pre-sized arena in a latency-critical server),
// and plug-in hosts that forbid cudaMalloc once they have started.
// rb_w8a8_gemm_noalloc runs the same GEMM as rb_w8a8_gemm_ws, taking its
// split-K workspace from the fixed device array below instead of from the
// caller.
//
// * The array lives for the life of the process on every GPU that loads this
//   library: kNoAllocScratchElems int32 = 20 MiB.  Any shape on a 148-SM B200
//   fits (the split heuristic never asks for more than 148 * 128 * 256 int32);
//   a shape that would need more is rejected with RB_ERR_VALUE.
// * The first call on a device looks up the array's device address with
//   cudaGetSymbolAddress (with that device current) and keeps it once the
//   lookup has succeeded (a failed lookup is retried by the next call); make
//   that first call before any stream capture that includes this entry point.
// * All calls share the one array.  Every partial a call reads was written
//   earlier in the same call, so nothing needs clearing between calls, but
//   two calls that run at the same time on the GPU (other streams, other host
//   threads) overwrite each other's partials: serialise them.
// * It calls no cudaMalloc, cudaFree or allocating library routine.
static constexpr int64_t kNoAllocScratchElems = 5 * 1024 * 1024;
static __device__ __align__(256) int32_t g_gemm_noalloc_scratch[kNoAllocScratchElems];
static int32_t* g_noalloc_scratch_ptr[64];  // the array's device address, once looked up
static std::mutex g_noalloc_scratch_mu;

extern "C" int rb_w8a8_gemm_noalloc(const int8_t* A, int64_t lda, const int8_t* B, int64_t ldb, int64_t M,
                                    int64_t N, int64_t K, const void* sa, int sa_dtype, int sa_per_row,
                                    const void* sb, int sb_dtype, const void* bias, int bias_dtype, void* out,
                                    int64_t ldo, int out_dtype, void* stream) {
  const int64_t need = rb_w8a8_gemm_workspace_size(M, N, K);
  if (need > kNoAllocScratchElems)
    return fail(RB_ERR_VALUE,
                "rb_w8a8_gemm_noalloc: M=%lld N=%lld K=%lld needs %lld int32 of split-K scratch, above the "
                "library's fixed %lld; use rb_w8a8_gemm_ws with a workspace",
                (long long)M, (long long)N, (long long)K, (long long)need, (long long)kNoAllocScratchElems);
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return check_cuda(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return fail(RB_ERR_UNSUPPORTED, "device index %d out of range", dev);
  int32_t* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_noalloc_scratch_mu);
    if (g_noalloc_scratch_ptr[dev] == nullptr) {
      void* p = nullptr;
      e = cudaGetSymbolAddress(&p, g_gemm_noalloc_scratch);
      if (e != cudaSuccess) return check_cuda(e, "cudaGetSymbolAddress(g_gemm_noalloc_scratch)");
      g_noalloc_scratch_ptr[dev] = static_cast<int32_t*>(p);
    }
    scratch = g_noalloc_scratch_ptr[dev];
  }
  return rb_w8a8_gemm_ws(A, lda, B, ldb, M, N, K, sa, sa_dtype, sa_per_row, sb, sb_dtype, bias, bias_dtype, out,
                         ldo, out_dtype, scratch, kNoAllocScratchElems, stream);
}
