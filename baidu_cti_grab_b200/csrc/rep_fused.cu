// rep_fused.cu -- K1: fused embedding-bag gather -> fp32 sum-pool -> concat ->
// LayerNorm -> int8 quantisation for the RepEncoder (sm_100a).
//
// Replaces, in one launch per batch, the reference's
//   models.py:27-34   28x (values.clamp(0, V-1); nn.EmbeddingBag(sum, padding_idx=0))
//   models.py:39-45   torch.cat(..., dim=1) + nn.LayerNorm(28*512)
//   quantization/w8a8_triton_kernels.py:41-64 / 23-38  dynamic / static int8 quantiser
// The concatenated [N, 14336] row never reaches HBM: one CTA owns one item,
// warp w owns slots 4w..4w+3, and lane l of a warp owns columns 8l..8l+7 and
// 256+8l..256+8l+7 of each of its slots (two 16-byte vectors of a bf16 row).
// The pooled row sits in shared memory in the row dtype (28 KB for bf16)
// between the statistics, the normalisation and the quantiser.  The LayerNorm
// statistics follow ATen's CUDA LayerNorm (the kernel the reference's
// nn.LayerNorm runs on the GPU): 128 Welford chains, chain c walking columns
// 4c..4c+3 of every slot in order, a shuffle-down tree per 32 chains and a
// fixed merge of the four groups, var = m2/H and rstd = rsqrtf(var + eps).
// Two warps run the 128 chains, two per lane in packed fp32 pairs.  Every
// floating-point step is an explicit round-to-nearest operation in the same
// order as ATen's, so mean, rstd, the LayerNorm row and the int8 row equal
// the reference's bit for bit.
//
// HBM traffic per item (bf16 table, k ids per slot): 28*k*1 KB of table rows
// + 28*k*8 B ids + 28*2*8 B offsets (4 B each with int32 indices) + 14336 B
// int8 + 4 B scale.
#include "common.cuh"

namespace rb {

constexpr int kSlotsPerWarp = 4;
constexpr int kMaxWarps = (RB_MAX_SLOTS + kSlotsPerWarp - 1) / kSlotsPerWarp;
#ifndef RB_K1_BF16_ROWS
#define RB_K1_BF16_ROWS 2
#endif
constexpr int kDim = 512;

// kGatherLnQuantPlain / kDenseLnQuantPlain: kGatherLnQuant / kDenseLnQuant with
// dynamic quantisation and no pooled or LayerNorm output (the RepEncoder forward
// and the slot-sharded path's second stage), their runtime options compiled out
enum RepMode : int {
  kGatherLnQuant = 0,
  kGatherPool = 1,
  kDenseLnQuant = 2,
  kGatherLnQuantPlain = 3,
  kDenseLnQuantPlain = 4
};

struct SlotArgs {
  // ids and offsets of each slot: int64, or int32 for the kernels instantiated
  // with IdxT = int32_t (the kernel reads them through IdxT)
  const void* values[RB_MAX_SLOTS];
  const void* offsets[RB_MAX_SLOTS];
  int64_t nnz[RB_MAX_SLOTS];
  int col_slot[RB_MAX_SLOTS];
};

struct RepParams {
  SlotArgs slots;
  const void* table;
  int64_t num_rows;
  const void* xs[RB_MAX_SLOTS];  // dense pooled rows (kDenseLnQuant): slot s of item i at xs[s] + i*ldx
  int64_t ldx;
  int num_slots;
  int64_t num_items;
  const void* gamma;
  const void* beta;
  int ln_dtype;
  int affine_v8;  // fp32 gamma/beta are 32-byte aligned: read with 256-bit loads
  float eps;
  int act_mode;
  const void* static_scale;
  int static_scale_dtype;
  int8_t* q;
  int64_t ldq;
  float* scale;
  void* pooled;
  int64_t ldp;
  void* ln;
  // pooling with scatter (num_dest > 0): item i with dest_begin[d] <= i < dest_begin[d+1]
  // goes to dest[d] + (i - dest_begin[d])*ldp, possibly another GPU's memory
  int num_dest;
  void* dest[RB_MAX_DEST];
  int64_t dest_begin[RB_MAX_DEST + 1];
  int64_t item_shift;  // CTA b pools item (b + item_shift) % num_items
};

// bf16 pair packed in a 32-bit word (lo element in the low half) -> fp32 pair
__device__ __forceinline__ F2 bf2(uint32_t w) { return f2(bf16_lo(w), bf16_hi(w)); }

// round_half_away_from_zero(v) for |v| < 2^23, exactly: the result is
// trunc(v + copysign(0.5, v)) with the addition rounded toward zero, because
// floor(RZ(|v| + 0.5)) == floor(|v| + 0.5) (every integer below 2^24 is
// representable, and rounding toward zero never crosses one downward).
__device__ __forceinline__ void round_half_away2(F2 v, int& q0, int& q1) {
  const float2 x = un(v);
  const F2 h = f2(__uint_as_float((__float_as_uint(x.x) & 0x80000000u) | 0x3f000000u),
                  __uint_as_float((__float_as_uint(x.y) & 0x80000000u) | 0x3f000000u));
  const float2 r = un(addrz2(v, h));
  q0 = __float2int_rz(r.x);
  q1 = __float2int_rz(r.y);
}

// four int32 values (each in [-128, 127]) as bytes a, b, c, d of one word:
// cvt.pack.sat puts its second operand in the low byte, its first in the next
// and the low 16 bits of its third above them
__device__ __forceinline__ uint32_t pack_i8x4_sat(int a, int b, int c, int d) {
  uint32_t hi, r;
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(hi) : "r"(d), "r"(c), "r"(0u));
  asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(b), "r"(a), "r"(hi));
  return r;
}

// running absmax of packed bf16 pairs: each half keeps max(|acc|, |w|) (the
// sign of the result is the xor of the operands' signs and is discarded)
__device__ __forceinline__ uint32_t absmax_bf16x2(uint32_t acc, uint32_t w) {
  uint32_t r;
  asm("max.xorsign.abs.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(acc), "r"(w));
  return r;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int d = 16; d >= 1; d >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, d));
  return v;
}

// ------------------------------------------ bf16 operands in fp32 arithmetic
// add/sub.rn.f32.bf16 widen a bf16 operand exactly and round the fp32 result
// once, i.e. they equal the fp32 op on the unpacked value without the unpack.
__device__ __forceinline__ float add_lo(float acc, uint32_t w) {
  float d;
  asm("{.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tadd.rn.f32.bf16 %0, lo, %2;\n\t}" : "=f"(d) : "r"(w), "f"(acc));
  return d;
}
__device__ __forceinline__ float add_hi(float acc, uint32_t w) {
  float d;
  asm("{.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tadd.rn.f32.bf16 %0, hi, %2;\n\t}" : "=f"(d) : "r"(w), "f"(acc));
  return d;
}
__device__ __forceinline__ float sub_lo(uint32_t w, float m) {  // bf16(lo) - m
  float d;
  asm("{.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tsub.rn.f32.bf16 %0, lo, %2;\n\t}" : "=f"(d) : "r"(w), "f"(m));
  return d;
}
__device__ __forceinline__ float sub_hi(uint32_t w, float m) {  // bf16(hi) - m
  float d;
  asm("{.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tsub.rn.f32.bf16 %0, hi, %2;\n\t}" : "=f"(d) : "r"(w), "f"(m));
  return d;
}

// ------------------------------------------------ row pieces per element type
// A lane's 16 values of a 512-wide slot segment are columns 8l..8l+7 and
// 256+8l..256+8l+7.  bf16 rows travel as 8 packed words (w[i] = elements
// 2i, 2i+1); fp32 rows as 8 fp32 pairs.
__device__ __forceinline__ void ldg_words(const void* seg, int lane, uint32_t* w) {
  const uint4* p = reinterpret_cast<const uint4*>(seg);
  const uint4 a = __ldg(p + lane), b = __ldg(p + 32 + lane);
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ void st_words(void* seg, int lane, const uint32_t* w) {
  uint4* p = reinterpret_cast<uint4*>(seg);
  p[lane] = make_uint4(w[0], w[1], w[2], w[3]);
  p[32 + lane] = make_uint4(w[4], w[5], w[6], w[7]);
}
__device__ __forceinline__ void ld_words(const void* seg, int lane, uint32_t* w) {  // shared or global, cached
  const uint4* p = reinterpret_cast<const uint4*>(seg);
  const uint4 a = p[lane], b = p[32 + lane];
  w[0] = a.x; w[1] = a.y; w[2] = a.z; w[3] = a.w;
  w[4] = b.x; w[5] = b.y; w[6] = b.z; w[7] = b.w;
}
__device__ __forceinline__ void ldg_pairs(const float* seg, int lane, F2* x) {
  const float4* p = reinterpret_cast<const float4*>(seg);
  const float4 a = __ldg(p + 2 * lane), b = __ldg(p + 2 * lane + 1), c = __ldg(p + 64 + 2 * lane),
               d = __ldg(p + 64 + 2 * lane + 1);
  x[0] = f2(a.x, a.y); x[1] = f2(a.z, a.w); x[2] = f2(b.x, b.y); x[3] = f2(b.z, b.w);
  x[4] = f2(c.x, c.y); x[5] = f2(c.z, c.w); x[6] = f2(d.x, d.y); x[7] = f2(d.z, d.w);
}
__device__ __forceinline__ void stg_pairs(float* seg, int lane, const F2* x) {
  float4* p = reinterpret_cast<float4*>(seg);
  const float2 v0 = un(x[0]), v1 = un(x[1]), v2 = un(x[2]), v3 = un(x[3]);
  const float2 v4 = un(x[4]), v5 = un(x[5]), v6 = un(x[6]), v7 = un(x[7]);
  p[2 * lane] = make_float4(v0.x, v0.y, v1.x, v1.y);
  p[2 * lane + 1] = make_float4(v2.x, v2.y, v3.x, v3.y);
  p[64 + 2 * lane] = make_float4(v4.x, v4.y, v5.x, v5.y);
  p[64 + 2 * lane + 1] = make_float4(v6.x, v6.y, v7.x, v7.y);
}
// fp32 row in shared memory, lane-major per slot (conflict-free 16-byte accesses):
// chunk c (0..3) of lane l of slot s = pairs 2c, 2c+1, at float s*512 + c*128 + 4l
__device__ __forceinline__ void sts_pairs(float* row, int s, int lane, const F2* x) {
  float4* p = reinterpret_cast<float4*>(row + s * kDim) + lane;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float2 u = un(x[2 * c]), v = un(x[2 * c + 1]);
    p[32 * c] = make_float4(u.x, u.y, v.x, v.y);
  }
}
__device__ __forceinline__ void lds_pairs(const float* row, int s, int lane, F2* x) {
  const float4* p = reinterpret_cast<const float4*>(row + s * kDim) + lane;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    const float4 v = p[32 * c];
    x[2 * c] = f2(v.x, v.y);
    x[2 * c + 1] = f2(v.z, v.w);
  }
}

// 8 fp32 values of 32 contiguous bytes (one 256-bit load; p 32-byte aligned)
__device__ __forceinline__ void ldg_v8(const float* p, float* v) {
  asm("ld.global.nc.v8.f32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=f"(v[0]), "=f"(v[1]), "=f"(v[2]), "=f"(v[3]), "=f"(v[4]), "=f"(v[5]), "=f"(v[6]), "=f"(v[7])
      : "l"(p));
}

// LayerNorm gamma and beta of one slot for one lane (its 16 columns), kept as
// loaded.  The lane's columns 8l..8l+7 and 256+8l..256+8l+7 are read as two
// contiguous pieces per tensor, so a warp reads each half-slot as one
// contiguous block: 16 bytes per lane for 16-bit parameters, 32 bytes (one
// 256-bit load, or two 128-bit loads when the tensors are only 16-byte
// aligned) for fp32 parameters.
template <typename TA>
struct Affine;

template <>
struct Affine<uint16_t> {  // bf16 or fp16 parameters (p.ln_dtype says which)
  uint32_t g[8], b[8];
  __device__ __forceinline__ void load(const RepParams& p, int s, int lane) {
    ldg_words(reinterpret_cast<const uint16_t*>(p.gamma) + s * kDim, lane, g);
    ldg_words(reinterpret_cast<const uint16_t*>(p.beta) + s * kDim, lane, b);
  }
  static __device__ __forceinline__ F2 widen(uint32_t w, bool bf) {
    if (bf) return bf2(w);
    const float2 h = __half22float2(*reinterpret_cast<const __half2*>(&w));
    return f2(h.x, h.y);
  }
  __device__ __forceinline__ F2 gamma(int i, bool bf) const { return widen(g[i], bf); }
  __device__ __forceinline__ F2 beta(int i, bool bf) const { return widen(b[i], bf); }
};

template <>
struct Affine<float> {
  float g[16], b[16];
  __device__ __forceinline__ void load(const RepParams& p, int s, int lane) {
    const float* gp = reinterpret_cast<const float*>(p.gamma) + s * kDim + 8 * lane;
    const float* bp = reinterpret_cast<const float*>(p.beta) + s * kDim + 8 * lane;
    if (p.affine_v8) {
      ldg_v8(gp, g);
      ldg_v8(gp + 256, g + 8);
      ldg_v8(bp, b);
      ldg_v8(bp + 256, b + 8);
    } else {
      ld4(gp, g); ld4(gp + 4, g + 4); ld4(gp + 256, g + 8); ld4(gp + 260, g + 12);
      ld4(bp, b); ld4(bp + 4, b + 4); ld4(bp + 256, b + 8); ld4(bp + 260, b + 12);
    }
  }
  static __device__ __forceinline__ void ld4(const float* p, float* v) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  }
  __device__ __forceinline__ F2 gamma(int i, bool) const { return f2(g[2 * i], g[2 * i + 1]); }
  __device__ __forceinline__ F2 beta(int i, bool) const { return f2(b[2 * i], b[2 * i + 1]); }
};

// Table rows of -0.0 (bf16 and fp32).  x + (-0.0) == x for every fp32 x (+0
// and -0 included), so a padding id, or a position past the end of a bag,
// reads this row and is added like any other instead of being branched around.
#define RB_NZ4 0x80008000u, 0x80008000u, 0x80008000u, 0x80008000u
#define RB_NZ16 RB_NZ4, RB_NZ4, RB_NZ4, RB_NZ4
#define RB_NZ64 RB_NZ16, RB_NZ16, RB_NZ16, RB_NZ16
static __device__ __align__(16) const uint32_t g_negzero_row_bf16[kDim / 2] = {RB_NZ64, RB_NZ64, RB_NZ64, RB_NZ64};
#define RB_NZF4 0x80000000u, 0x80000000u, 0x80000000u, 0x80000000u
#define RB_NZF16 RB_NZF4, RB_NZF4, RB_NZF4, RB_NZF4
#define RB_NZF64 RB_NZF16, RB_NZF16, RB_NZF16, RB_NZF16
#define RB_NZF256 RB_NZF64, RB_NZF64, RB_NZF64, RB_NZF64
static __device__ __align__(16) const uint32_t g_negzero_row_f32[kDim] = {RB_NZF256, RB_NZF256};
#undef RB_NZF256
#undef RB_NZF64
#undef RB_NZF16
#undef RB_NZF4
#undef RB_NZ64
#undef RB_NZ16
#undef RB_NZ4

__device__ __forceinline__ int32_t shfl_idx(int32_t v, int src) { return __shfl_sync(0xffffffffu, v, src); }
__device__ __forceinline__ int64_t shfl_idx(int64_t v, int src) {
  int lo = __shfl_sync(0xffffffffu, (int)(v & 0xffffffff), src);
  int hi = __shfl_sync(0xffffffffu, (int)(v >> 32), src);
  return ((int64_t)hi << 32) | (uint32_t)lo;
}

// a[j] for a runtime j in [0, N) without dynamic register indexing
template <int N, typename V>
__device__ __forceinline__ V sel(const V* a, int j) {
  V r = a[0];
#pragma unroll
  for (int i = 1; i < N; ++i)
    if (j == i) r = a[i];
  return r;
}

// ------------------------------------- LayerNorm statistics in ATen's order
// ATen's CUDA LayerNorm forward (PyTorch aten/src/ATen/native/cuda/
// layer_norm_kernel.cu: vectorized_layer_norm_kernel -> compute_stats,
// cuWelfordOnlineSum, cuWelfordCombine; 128 threads per row) keeps one
// Welford state per thread.  Thread c walks columns 4c..4c+3 of slot 0, then
// of slot 1, ... (groups of 4 elements strided by 128 groups); each warp's 32
// states are merged by shuffle-down (distances 16..1), then warps 0,1 merge
// warps 2,3 and warp 0 merges warp 1.  Here a lane of warps 0-1 carries
// chains c and c + 64 in the two halves of packed fp32 pairs.
struct Welford2 {
  F2 mean, m2;
};

// cuWelfordOnlineSum on both chains: r = 1/(count + 1), rounded once
__device__ __forceinline__ void welford_push2(Welford2& s, F2 x, float r) {
  const F2 delta = sub2(x, s.mean);
  s.mean = fma2(delta, f2(r, r), s.mean);
  s.m2 = fma2(delta, sub2(x, s.mean), s.m2);
}

// cuWelfordCombine(dataB = b, dataA = a) when both sides hold `cnt` elements:
// delta = b.mean - a.mean, nA = nB = cnt * (1 / (2 cnt)),
// mean = fma(nA, a.mean, nB * b.mean), m2 = fma(delta * delta * cnt, nB, a.m2 + b.m2)
__device__ __forceinline__ Welford2 welford_merge2(const Welford2& b, const Welford2& a, float cnt) {
  const float n = __fmul_rn(cnt, __fdiv_rn(1.0f, __fadd_rn(cnt, cnt)));
  const F2 n2 = f2(n, n);
  const F2 delta = sub2(b.mean, a.mean);
  Welford2 o;
  o.mean = fma2(n2, a.mean, mul2(n2, b.mean));
  o.m2 = fma2(mul2(mul2(delta, delta), f2(cnt, cnt)), n2, add2(a.m2, b.m2));
  return o;
}

__device__ __forceinline__ float2 welford_merge1(float b_mean, float b_m2, float a_mean, float a_m2, float cnt) {
  const float n = __fmul_rn(cnt, __fdiv_rn(1.0f, __fadd_rn(cnt, cnt)));
  const float delta = __fsub_rn(b_mean, a_mean);
  const float mean = __fmaf_rn(n, a_mean, __fmul_rn(n, b_mean));
  const float m2 = __fmaf_rn(__fmul_rn(__fmul_rn(delta, delta), cnt), n, __fadd_rn(a_m2, b_m2));
  return make_float2(mean, m2);
}

// One CTA per item.  Warp w owns slots 4w..4w+3 and lane l owns 16 columns
// of each (file header).  Per slot the warp sums the bag's table rows in bag
// order (kRows rows in flight; the rows of the warp's id window were already
// requested into L2, line by line) and rounds the sums to the row dtype
// into the item's shared-memory row.  After a barrier warps 0-1 run the 128
// LayerNorm chains of ATen's order over the row (lane l: chains l and l + 64 of
// its warp's half, as a packed fp32 pair) and leave two merged states in shared
// memory; after a second barrier every warp finishes the merge (mean, rstd)
// itself, normalises its slots in place (y rounded to the row dtype) with the
// absmax, and after a third barrier quantises them to int8.  bf16 rows stay
// packed in shared memory (28 KB per item) and enter fp32 arithmetic through
// the mixed-precision add/sub.  TA is the storage type of gamma/beta (uint16_t
// for bf16/fp16, float).  With bf16 rows the register budget (48 per thread)
// keeps five 7-warp CTAs resident per SM: the gather's latency, and the
// chains' serial tail (112 dependent Welford steps), need that occupancy more
// than the code needs registers.  An fp32 row takes 56 KB of shared memory, so
// at most three CTAs fit and the budget is larger.
template <typename T, int MODE, int kS, typename TA, typename IdxT>
__global__ void __launch_bounds__(256, sizeof(T) == 2 ? 5 : 3) rep_fused_kernel(const __grid_constant__ RepParams p) {
  constexpr bool kBf16 = sizeof(T) == 2;
  constexpr int kRows = kBf16 ? RB_K1_BF16_ROWS : 2;  // table rows a warp holds in registers
  extern __shared__ __align__(16) uint8_t s_raw[];
  __shared__ float s_stat[4];  // Welford (mean, m2) of chain groups {0,2} and {1,3}
  __shared__ float s_wmax[kMaxWarps];
  __shared__ const T* s_rowptr[kMaxWarps * 32];  // per pooling warp: row addresses of its id window
  uint32_t* s_words = reinterpret_cast<uint32_t*>(s_raw);  // bf16 row: 256 words per slot
  float* s_f32 = reinterpret_cast<float*>(s_raw);          // fp32 row: 512 floats per slot

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  constexpr bool kPlain = MODE == kGatherLnQuantPlain || MODE == kDenseLnQuantPlain;
  constexpr bool kDense = MODE == kDenseLnQuant || MODE == kDenseLnQuantPlain;
  const int64_t item =
      (kPlain || p.item_shift == 0) ? (int64_t)blockIdx.x : ((int64_t)blockIdx.x + p.item_shift) % p.num_items;
  // kS: the slot count when known at compile time (28 for the RepEncoder), else 0
  const int S = kS ? kS : p.num_slots;
  // warp w owns slots 4w .. 4w+3 (fewer in the last warp when S % 4 != 0)
  if (kS) __builtin_assume(warp < (kS + kSlotsPerWarp - 1) / kSlotsPerWarp);
  auto slot_of = [&](int j) { return warp * kSlotsPerWarp + j; };
  const int nsl = max(0, min(kSlotsPerWarp, S - warp * kSlotsPerWarp));
  // pooling modes: start of this item's output row (its own buffer, or the
  // receive buffer of the rank that owns the item)
  T* out_row = nullptr;
  if constexpr (MODE == kGatherPool) {
    if (p.num_dest == 0) {
      out_row = reinterpret_cast<T*>(p.pooled) + item * p.ldp;
    } else {
      int d = 0;
      while (d + 1 < p.num_dest && item >= p.dest_begin[d + 1]) ++d;
      out_row = reinterpret_cast<T*>(p.dest[d]) + (item - p.dest_begin[d]) * p.ldp;
    }
  }

  // the warp's j-th slot is pooled in `acc` (fp32, not yet rounded): round it
  // to T into shared memory (and the optional pooled output)
  auto finish_slot = [&](int j, const float* acc) {
    const int s = slot_of(j);
    if constexpr (kBf16) {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) w[i] = pack_bf16x2(acc[2 * i], acc[2 * i + 1]);
      st_words(s_words + s * 256, lane, w);
      if constexpr (MODE == kGatherPool) {
        if (p.num_dest == 0) st_words(out_row + (int64_t)p.slots.col_slot[s] * kDim, lane, w);
      } else if (!kPlain && p.pooled != nullptr) {
        st_words(reinterpret_cast<T*>(p.pooled) + item * p.ldp + (int64_t)s * kDim, lane, w);
      }
    } else {
      F2 x[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = f2(acc[2 * i], acc[2 * i + 1]);
      sts_pairs(s_f32, s, lane, x);
      if constexpr (MODE == kGatherPool) {
        stg_pairs(reinterpret_cast<float*>(out_row) + (int64_t)p.slots.col_slot[s] * kDim, lane, x);
      } else if (!kPlain && p.pooled != nullptr) {
        stg_pairs(reinterpret_cast<float*>(p.pooled) + item * p.ldp + (int64_t)s * kDim, lane, x);
      }
    }
  };

  if constexpr (kDense) {
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      if (j >= nsl) break;
      const T* xseg = reinterpret_cast<const T*>(p.xs[slot_of(j)]) + item * p.ldx;
      float acc[16];
      if constexpr (kBf16) {
        uint32_t w[8];
        ldg_words(xseg, lane, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          acc[2 * i] = bf16_lo(w[i]);
          acc[2 * i + 1] = bf16_hi(w[i]);
        }
      } else {
        F2 x[8];
        ldg_pairs(reinterpret_cast<const float*>(xseg), lane, x);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 v = un(x[i]);
          acc[2 * i] = v.x;
          acc[2 * i + 1] = v.y;
        }
      }
      finish_slot(j, acc);
    }
  } else {
    // ---- bag bounds of this warp's slots: lanes 0..3 starts, lanes 4..7 ends
    // bag positions fit the index type (int32 offsets address at most 2^31 ids)
    IdxT bound = 0;
    {
      const bool is_start = lane < kSlotsPerWarp;
      const int j = is_start ? lane : lane - kSlotsPerWarp;
      if (lane < 2 * kSlotsPerWarp && j < nsl) {
        const int s = slot_of(j);
        const int64_t nz = p.slots.nnz[s];
        const IdxT* off = static_cast<const IdxT*>(p.slots.offsets[s]);
        const int64_t b = is_start ? (int64_t)off[item] : ((item + 1 < p.num_items) ? (int64_t)off[item + 1] : nz);
        bound = (IdxT)(b < 0 ? 0 : (b > nz ? nz : b));
      }
    }
    // each bag's positions padded to a multiple of kRows: slot j of the warp
    // owns positions pre[j] .. pre[j+1]-1 of the warp's position list, its
    // first len[j] positions the bag's ids, the rest the -0.0 row
    IdxT start[kSlotsPerWarp];
    int len[kSlotsPerWarp];
    int pre[kSlotsPerWarp + 1];
    int total = 0;
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      start[j] = shfl_idx(bound, j);
      const IdxT e = shfl_idx(bound, kSlotsPerWarp + j);
      len[j] = (j < nsl && e > start[j]) ? (int)(e - start[j]) : 0;
      pre[j] = total;
      total += (len[j] + kRows - 1) / kRows * kRows;
    }
    pre[kSlotsPerWarp] = total;

    const T* table = reinterpret_cast<const T*>(p.table);
    const T* const pad_row = kBf16 ? reinterpret_cast<const T*>(g_negzero_row_bf16)
                                   : reinterpret_cast<const T*>(g_negzero_row_f32);
    const int vmax = (int)(p.num_rows - 1);
    // row addresses of positions w0 .. w0+31 into the warp's pointer list (one
    // per lane); each table row is requested into L2 as soon as its id is known
    const T** const wptr = s_rowptr + warp * 32;
    auto load_window = [&](int w0) {
      const int t = w0 + lane;
      const T* row = pad_row;
      if (t < total) {
        int j = 0;
#pragma unroll
        for (int i = 1; i < kSlotsPerWarp; ++i) j += t >= pre[i];
        const int k = t - sel<kSlotsPerWarp>(pre, j);
        if (k < sel<kSlotsPerWarp>(len, j)) {
          const int64_t v =
              static_cast<const IdxT*>(p.slots.values[slot_of(j)])[(int64_t)sel<kSlotsPerWarp>(start, j) + k];
          const int id = (int)(v < 0 ? 0 : (v > vmax ? vmax : v));
          if (id != 0) {
            row = table + (int64_t)id * kDim;
            // the row's 128-byte lines, one per-lane prefetch each: a bulk
            // prefetch takes one address per warp instruction, so 32 lanes'
            // rows cost 32 issues (7 more instructions per id, measured)
#pragma unroll
            for (int i = 0; i < kDim * (int)sizeof(T) / 128; ++i)
              asm volatile("prefetch.global.L2 [%0];" ::"l"(reinterpret_cast<const char*>(row) + 128 * i));
          }
        }
      }
      __syncwarp();  // every lane is done reading the previous window
      wptr[lane] = row;
      __syncwarp();
    };
    int w0 = 0;
    load_window(0);

#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      if (j >= nsl) break;
      const int tend = pre[j + 1];
      float acc[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) acc[e] = 0.0f;
      for (int t = pre[j]; t < tend; t += kRows) {
        if (t + kRows > w0 + 32) {  // warp-uniform: slide the window
          w0 = t;
          load_window(w0);
        }
        // the kRows row addresses (a broadcast read: every lane reads the same entries)
        const T* rows[kRows];
#pragma unroll
        for (int u = 0; u < kRows; ++u) rows[u] = wptr[t - w0 + u];
        if constexpr (kBf16) {
          uint32_t buf[kRows][8];
          // a padding id (0, or a negative id clamped to 0) and the positions past
          // the bag add the -0.0 row: no branch
#pragma unroll
          for (int u = 0; u < kRows; ++u) ldg_words(rows[u], lane, buf[u]);
#pragma unroll
          for (int u = 0; u < kRows; ++u) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              acc[2 * i] = add_lo(acc[2 * i], buf[u][i]);
              acc[2 * i + 1] = add_hi(acc[2 * i + 1], buf[u][i]);
            }
          }
        } else {
          F2 buf[kRows][8];
#pragma unroll
          for (int u = 0; u < kRows; ++u) ldg_pairs(reinterpret_cast<const float*>(rows[u]), lane, buf[u]);
#pragma unroll
          for (int u = 0; u < kRows; ++u) {
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const float2 v = un(buf[u][i]);
              acc[2 * i] = __fadd_rn(acc[2 * i], v.x);
              acc[2 * i + 1] = __fadd_rn(acc[2 * i + 1], v.y);
            }
          }
        }
      }
      finish_slot(j, acc);
    }
  }

  if constexpr (MODE == kGatherPool && kBf16) {
    if (p.num_dest > 0) {
      // scatter: the item's pooled bf16 row is complete in shared memory; copy
      // it to its owner 32 bytes per thread per step (a warp writes 1 KB per
      // store instruction), so the rows cross NVLink in whole sectors.  No
      // fence: the stores happen before the kernel's completion, which happens
      // before the caller's barrier (a collective on the same stream) whose
      // cross-GPU release/acquire publishes them to the owner.
      __syncthreads();
      for (int c = threadIdx.x; c < S * 32; c += blockDim.x) {
        const int s = c >> 5, k = c & 31;
        const uint4* src = reinterpret_cast<const uint4*>(s_words + s * 256) + 2 * k;
        const uint4 a = src[0], b = src[1];
        const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        stg_v8(out_row + (int64_t)p.slots.col_slot[s] * kDim + 16 * k, w);
      }
    }
  }
  if constexpr (MODE != kGatherPool) {
    const float H = (float)(S * kDim);
    const bool bf_affine = p.ln_dtype == RB_BF16;
    // the first slot's gamma/beta are requested before the barriers
    Affine<TA> aff;
    if (nsl > 0) aff.load(p, slot_of(0), lane);
    __syncthreads();  // the item's pooled row is complete in shared memory
    if (warp < 2) {
      // chains u and u + 64 of the 128 (u = threadIdx.x), as the halves of one pair
      const int u = threadIdx.x;
      Welford2 st{f2(0.0f, 0.0f), f2(0.0f, 0.0f)};
#pragma unroll
      for (int k = 0; k < RB_MAX_SLOTS; ++k) {
        if (k >= S) break;
        float lo[4], hi[4];
        if constexpr (kBf16) {
          const uint2 a = *reinterpret_cast<const uint2*>(s_words + k * 256 + 2 * u);
          const uint2 b = *reinterpret_cast<const uint2*>(s_words + k * 256 + 128 + 2 * u);
          lo[0] = bf16_lo(a.x); lo[1] = bf16_hi(a.x); lo[2] = bf16_lo(a.y); lo[3] = bf16_hi(a.y);
          hi[0] = bf16_lo(b.x); hi[1] = bf16_hi(b.x); hi[2] = bf16_lo(b.y); hi[3] = bf16_hi(b.y);
        } else {
          // fp32 rows are lane-major per slot (sts_pairs): columns 4u..4u+3 sit
          // at chunk u & 1 of lane u >> 1, columns 256 + 4u.. two chunks later
          const float* base = s_f32 + k * kDim + (u & 1) * 128 + 4 * (u >> 1);
          const float4 a = *reinterpret_cast<const float4*>(base);
          const float4 b = *reinterpret_cast<const float4*>(base + 256);
          lo[0] = a.x; lo[1] = a.y; lo[2] = a.z; lo[3] = a.w;
          hi[0] = b.x; hi[1] = b.y; hi[2] = b.z; hi[3] = b.w;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) welford_push2(st, f2(lo[e], hi[e]), 1.0f / (float)(4 * k + e + 1));
      }
      float cnt = (float)(4 * S);
#pragma unroll
      for (int d = 16; d >= 1; d >>= 1) {
        Welford2 o;
        o.mean.r = __shfl_down_sync(0xffffffffu, st.mean.r, d);
        o.m2.r = __shfl_down_sync(0xffffffffu, st.m2.r, d);
        st = welford_merge2(st, o, cnt);
        cnt = __fadd_rn(cnt, cnt);
      }
      if (lane == 0) {  // lo: chains of ATen warp `warp`, hi: of ATen warp `warp + 2`
        const float2 m = un(st.mean), q = un(st.m2);
        const float2 r = welford_merge1(m.x, q.x, m.y, q.y, cnt);
        s_stat[2 * warp] = r.x;
        s_stat[2 * warp + 1] = r.y;
      }
    }
    __syncthreads();
    float mean, rstd;
    {
      // ATen warp 0 (+2) merges warp 1 (+3); each side holds H / 2 elements
      const float2 r = welford_merge1(s_stat[0], s_stat[1], s_stat[2], s_stat[3], 0.5f * H);
      mean = r.x;
      const float var = __fdiv_rn(r.y, H);
      rstd = rsqrtf(__fadd_rn(var, p.eps));  // the CUDA function ATen's LayerNorm calls
    }
    const F2 mean2 = f2(mean, mean);
    const F2 rstd2 = f2(rstd, rstd);
    // ---- y = fma(rstd * (x - mean), gamma, beta) rounded to T, in place; absmax
    // (a rolled loop: the smaller code measured 2 % faster than four copies)
    float amax = 0.0f;
    uint32_t amax2 = 0u;  // bf16 rows: running absmax of the rounded pairs
#pragma unroll 1
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      if (j >= nsl) break;
      const int s = slot_of(j);
      if (j > 0) aff.load(p, s, lane);
      if constexpr (kBf16) {
        uint32_t w[8];
        ld_words(s_words + s * 256, lane, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const F2 d = f2(sub_lo(w[i], mean), sub_hi(w[i], mean));
          const float2 v = un(fma2(mul2(rstd2, d), aff.gamma(i, bf_affine), aff.beta(i, bf_affine)));
          w[i] = pack_bf16x2(v.x, v.y);
          // the quantiser's absmax is over the rounded row
          amax2 = absmax_bf16x2(amax2, w[i]);
        }
        st_words(s_words + s * 256, lane, w);
        if (!kPlain && p.ln != nullptr) st_words(reinterpret_cast<T*>(p.ln) + item * (int64_t)(S * kDim) + s * kDim, lane, w);
      } else {
        F2 x[8], y[8];
        lds_pairs(s_f32, s, lane, x);
#pragma unroll
        for (int i = 0; i < 8; ++i)
          y[i] = fma2(mul2(rstd2, sub2(x[i], mean2)), aff.gamma(i, bf_affine), aff.beta(i, bf_affine));
        sts_pairs(s_f32, s, lane, y);
        if (!kPlain && p.ln != nullptr) stg_pairs(reinterpret_cast<float*>(p.ln) + item * (int64_t)(S * kDim) + s * kDim, lane, y);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float2 v = un(y[i]);
          amax = fmaxf(amax, fmaxf(fabsf(v.x), fabsf(v.y)));
        }
      }
    }
    if (!kPlain && p.act_mode == RB_ACT_NONE) return;
    if constexpr (kBf16) amax = fmaxf(fabsf(bf16_lo(amax2)), fabsf(bf16_hi(amax2)));
    amax = warp_max(amax);
    if (lane == 0) s_wmax[warp] = amax;
    __syncthreads();
    // every thread derives the quantiser scale (no further barrier)
    float inv;
    if (kPlain || p.act_mode == RB_ACT_DYNAMIC) {
      float m = 0.0f;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, s_wmax[w]);
      m = fmaxf(m, 1e-8f);
      inv = __fdiv_rn(127.0f, m);
      if (threadIdx.x == 0) p.scale[item] = __fdiv_rn(m, 127.0f);
    } else {
      inv = __fdiv_rn(1.0f, load_as_f32(p.static_scale, p.static_scale_dtype, 0));
    }
    const F2 inv2 = f2(inv, inv);
    int8_t* const q_lane = p.q + item * p.ldq + 8 * lane;  // this lane's columns of the item's int8 row
    const bool clamp = !kPlain && p.act_mode == RB_ACT_STATIC;
    // ---- int8 = clamp(round_half_away(y * inv), -128, 127)
#pragma unroll
    for (int j = 0; j < kSlotsPerWarp; ++j) {
      if (j >= nsl) break;
      const int s = slot_of(j);
      F2 x[8];
      if constexpr (kBf16) {
        uint32_t w[8];
        ld_words(s_words + s * 256, lane, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) x[i] = bf2(w[i]);
      } else {
        lds_pairs(s_f32, s, lane, x);
      }
      int q[16];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        F2 v = mul2(x[i], inv2);
        if (clamp) {
          // |y*inv| <= 127*(1+2^-23) in dynamic mode; a static scale needs the clamp
          const float2 c = un(v);
          v = f2(fminf(fmaxf(c.x, -128.0f), 127.0f), fminf(fmaxf(c.y, -128.0f), 127.0f));
        }
        round_half_away2(v, q[2 * i], q[2 * i + 1]);
      }
      int8_t* dst = q_lane + s * kDim;
      *reinterpret_cast<uint2*>(dst) = make_uint2(pack_i8x4_sat(q[0], q[1], q[2], q[3]),
                                                  pack_i8x4_sat(q[4], q[5], q[6], q[7]));
      *reinterpret_cast<uint2*>(dst + 256) = make_uint2(pack_i8x4_sat(q[8], q[9], q[10], q[11]),
                                                        pack_i8x4_sat(q[12], q[13], q[14], q[15]));
    }
  }
}

// ------------------------------------------------------------------ host
static int validate_common(int num_slots, int64_t num_items) {
  if (num_slots < 1 || num_slots > RB_MAX_SLOTS)
    return fail(RB_ERR_VALUE, "num_slots must be in [1, %d], got %d", RB_MAX_SLOTS, num_slots);
  if (num_items < 0) return fail(RB_ERR_VALUE, "num_items must be >= 0");
  if (num_items > 0x7fffffffLL) return fail(RB_ERR_UNSUPPORTED, "num_items above 2^31-1 per call");
  return RB_OK;
}

static int fill_slots(SlotArgs& sa, const void* const* values, const void* const* offsets,
                      const int64_t* nnz, const int* col_slot, int num_slots, int64_t num_items) {
  for (int s = 0; s < num_slots; ++s) {
    if (offsets == nullptr || offsets[s] == nullptr)
      return fail(RB_ERR_VALUE, "slot %d: offsets pointer is null", s);
    if (nnz[s] < 0) return fail(RB_ERR_VALUE, "slot %d: nnz must be >= 0", s);
    if (nnz[s] > 0 && (values == nullptr || values[s] == nullptr))
      return fail(RB_ERR_VALUE, "slot %d: values pointer is null", s);
    sa.values[s] = values ? values[s] : nullptr;
    sa.offsets[s] = offsets[s];
    sa.nnz[s] = nnz[s];
    sa.col_slot[s] = col_slot ? col_slot[s] : s;
  }
  (void)num_items;
  return RB_OK;
}

template <int MODE, typename IdxT = int64_t>
static int launch_rep(const RepParams& p, int row_dtype, cudaStream_t stream) {
  if (p.num_items == 0) return RB_OK;
  // a warp per 4 slots, and at least the 2 warps that run the LayerNorm chains
  const int warps = max(2, (p.num_slots + kSlotsPerWarp - 1) / kSlotsPerWarp);
  dim3 grid((unsigned)p.num_items), block(32 * warps);
  // the item's pooled row: packed bf16, or fp32 for fp32 tables
  const size_t smem = (size_t)p.num_slots * kDim * dtype_size(row_dtype);
  cudaError_t e = cudaSuccess;
  // the RepEncoder's 28 slots get a specialised kernel
  const bool s28 = p.num_slots == 28;
  // gamma/beta storage: 16-bit words or fp32 (the pooling-only mode reads neither)
  const bool a16 = MODE != kGatherPool && p.ln_dtype != RB_F32;
  using B16 = __nv_bfloat16;
  auto kern = row_dtype == RB_BF16
                  ? (s28 ? (a16 ? rep_fused_kernel<B16, MODE, 28, uint16_t, IdxT>
                                : rep_fused_kernel<B16, MODE, 28, float, IdxT>)
                         : (a16 ? rep_fused_kernel<B16, MODE, 0, uint16_t, IdxT>
                                : rep_fused_kernel<B16, MODE, 0, float, IdxT>))
                  : (s28 ? (a16 ? rep_fused_kernel<float, MODE, 28, uint16_t, IdxT>
                                : rep_fused_kernel<float, MODE, 28, float, IdxT>)
                         : (a16 ? rep_fused_kernel<float, MODE, 0, uint16_t, IdxT>
                                : rep_fused_kernel<float, MODE, 0, float, IdxT>));
  if (smem > 48 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess) kern<<<grid, block, smem, stream>>>(p);
  if (e != cudaSuccess) return check_cuda(e, "cudaFuncSetAttribute(rep_fused_kernel)");
  return check_cuda(cudaGetLastError(), "rep_fused_kernel launch");
}

static int check_ln_args(const void* gamma, const void* beta, int ln_dtype, int act_mode,
                         const void* static_scale, int ss_dtype, const int8_t* q, int64_t ldq,
                         const float* scale, const void* ln_out, int num_slots) {
  if (gamma == nullptr || beta == nullptr) return fail(RB_ERR_VALUE, "LayerNorm gamma/beta must be given");
  if (ln_dtype != RB_BF16 && ln_dtype != RB_F32 && ln_dtype != RB_F16)
    return fail(RB_ERR_VALUE, "ln_dtype must be RB_BF16, RB_F16 or RB_F32");
  if (!aligned(gamma, 16) || !aligned(beta, 16)) return fail(RB_ERR_VALUE, "gamma/beta must be 16-byte aligned");
  if (act_mode == RB_ACT_DYNAMIC || act_mode == RB_ACT_STATIC) {
    if (q == nullptr) return fail(RB_ERR_VALUE, "q_out must be given");
    if (!aligned(q, 16) || ldq % 16 != 0 || ldq < (int64_t)num_slots * kDim)
      return fail(RB_ERR_VALUE, "q_out must be 16-byte aligned with ldq %% 16 == 0 and ldq >= %d",
                  num_slots * kDim);
    if (act_mode == RB_ACT_DYNAMIC && scale == nullptr) return fail(RB_ERR_VALUE, "scale_out must be given");
    if (act_mode == RB_ACT_STATIC) {
      if (static_scale == nullptr) return fail(RB_ERR_VALUE, "static_scale must be given");
      if (ss_dtype != RB_F32 && ss_dtype != RB_BF16 && ss_dtype != RB_F16)
        return fail(RB_ERR_VALUE, "static_scale dtype must be f32/bf16/f16");
    }
  } else if (act_mode == RB_ACT_NONE) {
    if (ln_out == nullptr) return fail(RB_ERR_VALUE, "act_mode RB_ACT_NONE needs ln_out");
  } else {
    return fail(RB_ERR_VALUE, "unknown act_mode %d", act_mode);
  }
  if (ln_out != nullptr && !aligned(ln_out, 16)) return fail(RB_ERR_VALUE, "ln_out must be 16-byte aligned");
  return RB_OK;
}

}  // namespace rb

using namespace rb;

static int gather_ln_quant(const void* table, int table_dtype, int64_t num_rows, int emb_dim, int index_dtype,
                           const void* const* slot_values, const void* const* slot_offsets,
                           const int64_t* slot_nnz, int num_slots, int64_t num_items, const void* ln_gamma,
                           const void* ln_beta, int ln_dtype, float eps, int act_mode, const void* static_scale,
                           int static_scale_dtype, int8_t* q_out, int64_t ldq, float* scale_out, void* pooled_out,
                           void* ln_out, void* stream) {
  if (index_dtype != RB_I64 && index_dtype != RB_I32)
    return fail(RB_ERR_VALUE, "index dtype must be RB_I64 or RB_I32, got %d", index_dtype);
  int rc = validate_common(num_slots, num_items);
  if (rc) return rc;
  if (emb_dim != kDim) return fail(RB_ERR_UNSUPPORTED, "emb_dim must be 512, got %d", emb_dim);
  if (table_dtype != RB_BF16 && table_dtype != RB_F32)
    return fail(RB_ERR_VALUE, "table dtype must be RB_BF16 or RB_F32");
  if (table == nullptr || !aligned(table, 16)) return fail(RB_ERR_VALUE, "table must be 16-byte aligned");
  if (num_rows < 1 || num_rows > 0x7fffffffLL)
    return fail(RB_ERR_VALUE, "num_rows must be in [1, 2^31-1] (ids are clamped in 32 bits), got %lld",
                (long long)num_rows);
  if (slot_nnz == nullptr) return fail(RB_ERR_VALUE, "slot_nnz must be given");
  if (num_items == 0) return RB_OK;  // empty batch: nothing to read or write
  rc = check_ln_args(ln_gamma, ln_beta, ln_dtype, act_mode, static_scale, static_scale_dtype, q_out, ldq,
                     scale_out, ln_out, num_slots);
  if (rc) return rc;
  if (pooled_out != nullptr && !aligned(pooled_out, 16))
    return fail(RB_ERR_VALUE, "pooled_out must be 16-byte aligned");
  RepParams p{};
  rc = fill_slots(p.slots, slot_values, slot_offsets, slot_nnz, nullptr, num_slots, num_items);
  if (rc) return rc;
  p.table = table;
  p.num_rows = num_rows;
  p.num_slots = num_slots;
  p.num_items = num_items;
  p.gamma = ln_gamma;
  p.beta = ln_beta;
  p.affine_v8 = aligned(ln_gamma, 32) && aligned(ln_beta, 32);
  p.ln_dtype = ln_dtype;
  p.eps = eps;
  p.act_mode = act_mode;
  p.static_scale = static_scale;
  p.static_scale_dtype = static_scale_dtype;
  p.q = q_out;
  p.ldq = ldq;
  p.scale = scale_out;
  p.pooled = pooled_out;
  p.ldp = (int64_t)num_slots * kDim;
  p.ln = ln_out;
  if (pooled_out == nullptr && ln_out == nullptr && act_mode == RB_ACT_DYNAMIC)
    return index_dtype == RB_I32 ? launch_rep<kGatherLnQuantPlain, int32_t>(p, table_dtype, (cudaStream_t)stream)
                                 : launch_rep<kGatherLnQuantPlain, int64_t>(p, table_dtype, (cudaStream_t)stream);
  return index_dtype == RB_I32 ? launch_rep<kGatherLnQuant, int32_t>(p, table_dtype, (cudaStream_t)stream)
                               : launch_rep<kGatherLnQuant, int64_t>(p, table_dtype, (cudaStream_t)stream);
}

extern "C" int rb_rep_gather_ln_quant(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                                      const int64_t* const* slot_values, const int64_t* const* slot_offsets,
                                      const int64_t* slot_nnz, int num_slots, int64_t num_items,
                                      const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps,
                                      int act_mode, const void* static_scale, int static_scale_dtype,
                                      int8_t* q_out, int64_t ldq, float* scale_out, void* pooled_out,
                                      void* ln_out, void* stream) {
  return gather_ln_quant(table, table_dtype, num_rows, emb_dim, RB_I64,
                         reinterpret_cast<const void* const*>(slot_values),
                         reinterpret_cast<const void* const*>(slot_offsets), slot_nnz, num_slots, num_items,
                         ln_gamma, ln_beta, ln_dtype, eps, act_mode, static_scale, static_scale_dtype, q_out, ldq,
                         scale_out, pooled_out, ln_out, stream);
}

extern "C" int rb_rep_gather_ln_quant_idx(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                                          int index_dtype, const void* const* slot_values,
                                          const void* const* slot_offsets, const int64_t* slot_nnz,
                                          int num_slots, int64_t num_items, const void* ln_gamma,
                                          const void* ln_beta, int ln_dtype, float eps, int act_mode,
                                          const void* static_scale, int static_scale_dtype, int8_t* q_out,
                                          int64_t ldq, float* scale_out, void* pooled_out, void* ln_out,
                                          void* stream) {
  return gather_ln_quant(table, table_dtype, num_rows, emb_dim, index_dtype, slot_values, slot_offsets, slot_nnz,
                         num_slots, num_items, ln_gamma, ln_beta, ln_dtype, eps, act_mode, static_scale,
                         static_scale_dtype, q_out, ldq, scale_out, pooled_out, ln_out, stream);
}

extern "C" int rb_rep_gather_pool(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                                  const int64_t* const* slot_values, const int64_t* const* slot_offsets,
                                  const int64_t* slot_nnz, const int* col_slot, int num_slots,
                                  int64_t num_items, void* pooled_out, int64_t ldp, void* stream) {
  int rc = validate_common(num_slots, num_items);
  if (rc) return rc;
  if (emb_dim != kDim) return fail(RB_ERR_UNSUPPORTED, "emb_dim must be 512, got %d", emb_dim);
  if (table_dtype != RB_BF16 && table_dtype != RB_F32)
    return fail(RB_ERR_VALUE, "table dtype must be RB_BF16 or RB_F32");
  if (table == nullptr || !aligned(table, 16)) return fail(RB_ERR_VALUE, "table must be 16-byte aligned");
  if (num_rows < 1 || num_rows > 0x7fffffffLL)
    return fail(RB_ERR_VALUE, "num_rows must be in [1, 2^31-1] (ids are clamped in 32 bits), got %lld",
                (long long)num_rows);
  if (slot_nnz == nullptr || col_slot == nullptr) return fail(RB_ERR_VALUE, "slot_nnz/col_slot must be given");
  if (num_items == 0) return RB_OK;
  if (pooled_out == nullptr || !aligned(pooled_out, 16))
    return fail(RB_ERR_VALUE, "pooled_out must be 16-byte aligned");
  const int esz = dtype_size(table_dtype);
  if ((ldp * esz) % 16 != 0) return fail(RB_ERR_VALUE, "ldp must keep rows 16-byte aligned");
  for (int s = 0; s < num_slots; ++s)
    if (col_slot[s] < 0 || (int64_t)(col_slot[s] + 1) * kDim > ldp)
      return fail(RB_ERR_VALUE, "col_slot[%d]=%d does not fit in ldp=%lld", s, col_slot[s], (long long)ldp);
  RepParams p{};
  rc = fill_slots(p.slots, reinterpret_cast<const void* const*>(slot_values),
                  reinterpret_cast<const void* const*>(slot_offsets), slot_nnz, col_slot, num_slots, num_items);
  if (rc) return rc;
  p.table = table;
  p.num_rows = num_rows;
  p.num_slots = num_slots;
  p.num_items = num_items;
  p.pooled = pooled_out;
  p.ldp = ldp;
  return launch_rep<kGatherPool>(p, table_dtype, (cudaStream_t)stream);
}

extern "C" int rb_rep_gather_pool_scatter(const void* table, int table_dtype, int64_t num_rows, int emb_dim,
                                          const int64_t* const* slot_values, const int64_t* const* slot_offsets,
                                          const int64_t* slot_nnz, const int* col_slot, int num_slots,
                                          int64_t num_items, void* const* dest, const int64_t* dest_begin,
                                          int num_dest, int64_t ld, int64_t item_shift, void* stream) {
  int rc = validate_common(num_slots, num_items);
  if (rc) return rc;
  if (emb_dim != kDim) return fail(RB_ERR_UNSUPPORTED, "emb_dim must be 512, got %d", emb_dim);
  if (table_dtype != RB_BF16 && table_dtype != RB_F32)
    return fail(RB_ERR_VALUE, "table dtype must be RB_BF16 or RB_F32");
  if (table == nullptr || !aligned(table, 16)) return fail(RB_ERR_VALUE, "table must be 16-byte aligned");
  if (num_rows < 1 || num_rows > 0x7fffffffLL)
    return fail(RB_ERR_VALUE, "num_rows must be in [1, 2^31-1] (ids are clamped in 32 bits), got %lld",
                (long long)num_rows);
  if (slot_nnz == nullptr || col_slot == nullptr) return fail(RB_ERR_VALUE, "slot_nnz/col_slot must be given");
  if (num_dest < 1 || num_dest > RB_MAX_DEST)
    return fail(RB_ERR_VALUE, "num_dest must be in [1, %d], got %d", RB_MAX_DEST, num_dest);
  if (dest == nullptr || dest_begin == nullptr) return fail(RB_ERR_VALUE, "dest/dest_begin must be given");
  if (dest_begin[0] != 0 || dest_begin[num_dest] != num_items)
    return fail(RB_ERR_VALUE, "dest_begin must run from 0 to num_items");
  const int esz = dtype_size(table_dtype);
  // bf16 rows leave in 32-byte stores, fp32 rows in 16-byte stores
  const int row_align = table_dtype == RB_BF16 ? 32 : 16;
  if ((ld * esz) % row_align != 0) return fail(RB_ERR_VALUE, "ld must keep rows %d-byte aligned", row_align);
  for (int d = 0; d < num_dest; ++d) {
    if (dest_begin[d + 1] < dest_begin[d]) return fail(RB_ERR_VALUE, "dest_begin must not decrease");
    if (dest_begin[d + 1] > dest_begin[d] && (dest[d] == nullptr || !aligned(dest[d], row_align)))
      return fail(RB_ERR_VALUE, "dest[%d] must be a %d-byte aligned pointer", d, row_align);
  }
  for (int s = 0; s < num_slots; ++s)
    if (col_slot[s] < 0 || (int64_t)(col_slot[s] + 1) * kDim > ld)
      return fail(RB_ERR_VALUE, "col_slot[%d]=%d does not fit in ld=%lld", s, col_slot[s], (long long)ld);
  if (num_items == 0) return RB_OK;
  if (item_shift < 0 || item_shift >= num_items) return fail(RB_ERR_VALUE, "item_shift must be in [0, num_items)");
  RepParams p{};
  rc = fill_slots(p.slots, reinterpret_cast<const void* const*>(slot_values),
                  reinterpret_cast<const void* const*>(slot_offsets), slot_nnz, col_slot, num_slots, num_items);
  if (rc) return rc;
  p.table = table;
  p.num_rows = num_rows;
  p.num_slots = num_slots;
  p.num_items = num_items;
  p.ldp = ld;
  p.item_shift = item_shift;
  p.num_dest = num_dest;
  for (int d = 0; d < num_dest; ++d) {
    p.dest[d] = dest[d];
    p.dest_begin[d] = dest_begin[d];
  }
  p.dest_begin[num_dest] = dest_begin[num_dest];
  return launch_rep<kGatherPool>(p, table_dtype, (cudaStream_t)stream);
}

static int layernorm_quant_common(RepParams& p, int x_dtype, int64_t num_items, int num_slots, int64_t ldx,
                                  const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps, int act_mode,
                                  const void* static_scale, int static_scale_dtype, int8_t* q_out, int64_t ldq,
                                  float* scale_out, void* ln_out, void* stream) {
  int rc = check_ln_args(ln_gamma, ln_beta, ln_dtype, act_mode, static_scale, static_scale_dtype, q_out, ldq,
                         scale_out, ln_out, num_slots);
  if (rc) return rc;
  p.ldx = ldx;
  p.num_slots = num_slots;
  p.num_items = num_items;
  p.gamma = ln_gamma;
  p.beta = ln_beta;
  p.affine_v8 = aligned(ln_gamma, 32) && aligned(ln_beta, 32);
  p.ln_dtype = ln_dtype;
  p.eps = eps;
  p.act_mode = act_mode;
  p.static_scale = static_scale;
  p.static_scale_dtype = static_scale_dtype;
  p.q = q_out;
  p.ldq = ldq;
  p.scale = scale_out;
  p.ln = ln_out;
  if (ln_out == nullptr && act_mode == RB_ACT_DYNAMIC) return launch_rep<kDenseLnQuantPlain>(p, x_dtype, (cudaStream_t)stream);
  return launch_rep<kDenseLnQuant>(p, x_dtype, (cudaStream_t)stream);
}

extern "C" int rb_layernorm_quant(const void* x, int x_dtype, int64_t num_items, int num_slots, int64_t ldx,
                                  const void* ln_gamma, const void* ln_beta, int ln_dtype, float eps,
                                  int act_mode, const void* static_scale, int static_scale_dtype,
                                  int8_t* q_out, int64_t ldq, float* scale_out, void* ln_out, void* stream) {
  int rc = validate_common(num_slots, num_items);
  if (rc) return rc;
  if (x_dtype != RB_BF16 && x_dtype != RB_F32) return fail(RB_ERR_VALUE, "x dtype must be RB_BF16 or RB_F32");
  if (num_items == 0) return RB_OK;
  const int esz = dtype_size(x_dtype);
  if (x == nullptr || !aligned(x, 16) || (ldx * esz) % 16 != 0 || ldx < (int64_t)num_slots * kDim)
    return fail(RB_ERR_VALUE, "x must be 16-byte aligned with 16-byte row stride and ldx >= %d",
                num_slots * kDim);
  RepParams p{};
  for (int s = 0; s < num_slots; ++s) p.xs[s] = reinterpret_cast<const char*>(x) + (int64_t)s * kDim * esz;
  return layernorm_quant_common(p, x_dtype, num_items, num_slots, ldx, ln_gamma, ln_beta, ln_dtype, eps, act_mode,
                                static_scale, static_scale_dtype, q_out, ldq, scale_out, ln_out, stream);
}

extern "C" int rb_layernorm_quant_slots(const void* const* slot_rows, int x_dtype, int64_t num_items,
                                        int num_slots, int64_t ld, const void* ln_gamma, const void* ln_beta,
                                        int ln_dtype, float eps, int act_mode, const void* static_scale,
                                        int static_scale_dtype, int8_t* q_out, int64_t ldq, float* scale_out,
                                        void* ln_out, void* stream) {
  int rc = validate_common(num_slots, num_items);
  if (rc) return rc;
  if (x_dtype != RB_BF16 && x_dtype != RB_F32) return fail(RB_ERR_VALUE, "x dtype must be RB_BF16 or RB_F32");
  if (num_items == 0) return RB_OK;
  const int esz = dtype_size(x_dtype);
  if (slot_rows == nullptr || (ld * esz) % 16 != 0 || ld < kDim)
    return fail(RB_ERR_VALUE, "slot rows need a 16-byte row stride ld >= 512");
  RepParams p{};
  for (int s = 0; s < num_slots; ++s) {
    if (slot_rows[s] == nullptr || !aligned(slot_rows[s], 16))
      return fail(RB_ERR_VALUE, "slot %d rows must be 16-byte aligned", s);
    p.xs[s] = slot_rows[s];
  }
  return layernorm_quant_common(p, x_dtype, num_items, num_slots, ld, ln_gamma, ln_beta, ln_dtype, eps, act_mode,
                                static_scale, static_scale_dtype, q_out, ldq, scale_out, ln_out, stream);
}
