// moe.cu -- the SMoE expert layer of the reference's TransformerEncoder
// (models.py:96-178, SMoE.forward after the gate) on sm_100a.
//
// Given the gate's top-k experts and scores of T tokens (R = T*k routed
// entries), the reference sorts the entries by expert, packs them into a
// zero-padded [E, max_count, D] block (sized by a host read of the largest
// count, models.py:160), runs two bmm's with the stacked expert weights and
// scatters the score-weighted rows back with index_add_.  Here:
//
//   route_count_kernel     per chunk of 256 entries, how many go to each expert
//   route_scatter_kernel   stable counting sort (the order of
//                          torch.argsort(stable=True)): expert offsets, the
//                          sorted entry list, and the packed rows
//                          packed[p] = x[entry / k] of each expert's segment
//   moe_gemm_pair_kernel<1>  per expert segment, hidden = relu(x W1^T + b1)
//   moe_gemm_pair_kernel<2>  per expert segment, y[entry] = (h W2^T + b2) * score
//   combine_kernel         out[t] = y[t*k] + y[t*k+1] + ... in slot order
//
// The grouped GEMMs read the expert offsets on the device: a persistent CTA
// pair walks tiles (expert, 256-row block, 256-column block) until the last
// expert's rows are covered, so nothing is read back by the host and no row
// of padding is multiplied.  They follow the CTA-pair tcgen05 pipeline of
// gemm_tc.cu (TMA -> 6-stage ring per CTA -> kind::f16 MMA of the pair into
// two 256x256 fp32 TMEM accumulators -> epilogue warps), with a per-tile B row
// offset of expert * N.  Rows of a 256-row block past its expert's segment are
// computed and discarded.
//
// Rounding follows the reference's bf16/fp16 torch ops step by step: the bmm
// result rounded to the model dtype, + bias (rounded), relu; the second bmm
// rounded, + bias (rounded), * score (rounded); index_add_ into zeros, which
// for the reference's k = 2 is the rounded sum of the two rows in either
// order.  Only the fp32 accumulation order inside each dot product differs
// from cuBLAS's.
#include "common.cuh"

#include <type_traits>

namespace rb {
namespace moe {

constexpr int kMaxExperts = 64;
constexpr int kRouteThreads = 256;
constexpr int kRouteChunk = 256;  // entries per CTA (one round of kRouteThreads): enough CTAs to fill the SMs
constexpr int kMoeBadExpert = 301;  // watchdog code: an expert id outside [0, E)

template <typename IdxT>
__device__ __forceinline__ int expert_of(const IdxT* idx, int64_t j, int64_t R, int E) {
  if (j >= R) return -1;
  const int64_t v = (int64_t)idx[j];
  if (v < 0 || v >= E) {
    raise_device_error(kMoeBadExpert);
    return -1;
  }
  return (int)v;
}

template <typename IdxT>
__global__ void __launch_bounds__(kRouteThreads) route_count_kernel(const IdxT* __restrict__ idx, int64_t R, int E,
                                                                    int32_t* __restrict__ chunk_hist) {
  __shared__ int hist[kMaxExperts];
  for (int e = threadIdx.x; e < E; e += blockDim.x) hist[e] = 0;
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int64_t base = (int64_t)blockIdx.x * kRouteChunk;
  for (int i = threadIdx.x; i < kRouteChunk; i += kRouteThreads) {
    const int e = expert_of(idx, base + i, R, E);
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0 && lane == __ffs(peers) - 1) atomicAdd(&hist[e], __popc(peers));
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) chunk_hist[(int64_t)blockIdx.x * E + e] = hist[e];
}

// Rows are copied 16 bytes per lane; row_bytes is a multiple of 16.
template <typename IdxT>
__global__ void __launch_bounds__(kRouteThreads) route_scatter_kernel(
    const IdxT* __restrict__ idx, int64_t R, int k, int E, int nchunks, const int32_t* __restrict__ chunk_hist,
    int32_t* __restrict__ offsets, int32_t* __restrict__ sorted_entry, const uint8_t* __restrict__ x,
    int64_t x_pitch, int64_t row_bytes, uint8_t* __restrict__ packed) {
  constexpr int kWarps = kRouteThreads / 32;
  __shared__ int s_before[kMaxExperts], s_total[kMaxExperts], s_off[kMaxExperts + 1], s_next[kMaxExperts];
  __shared__ int s_wcnt[kWarps][kMaxExperts];
  __shared__ int s_pos[kRouteThreads];
  __shared__ int64_t s_tok[kRouteThreads];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // where this chunk's rows of each expert start: the expert's offset plus
  // the rows that earlier chunks send to it
  for (int e = warp; e < E; e += kWarps) {
    int before = 0, total = 0;
    for (int c = lane; c < nchunks; c += 32) {
      const int h = chunk_hist[(int64_t)c * E + e];
      total += h;
      if (c < (int)blockIdx.x) before += h;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      before += __shfl_xor_sync(0xffffffffu, before, o);
      total += __shfl_xor_sync(0xffffffffu, total, o);
    }
    if (lane == 0) {
      s_before[e] = before;
      s_total[e] = total;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int off = 0;
    for (int e = 0; e < E; ++e) {
      s_off[e] = off;
      off += s_total[e];
    }
    s_off[E] = off;
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) s_next[e] = s_off[e] + s_before[e];
  if (blockIdx.x == 0)
    for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = s_off[e];

  const int64_t chunk0 = (int64_t)blockIdx.x * kRouteChunk;
  const int chunks16 = (int)(row_bytes / 16);
  for (int r = 0; r < kRouteChunk / kRouteThreads; ++r) {
    const int64_t j = chunk0 + r * kRouteThreads + threadIdx.x;
    __syncthreads();  // the previous round has read s_wcnt, s_pos and s_tok
    for (int i = threadIdx.x; i < kWarps * E; i += kRouteThreads) s_wcnt[i / E][i % E] = 0;
    __syncthreads();
    const int e = expert_of(idx, j, R, E);
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    const int rank = __popc(peers & ((1u << lane) - 1u));
    if (e >= 0 && lane == __ffs(peers) - 1) s_wcnt[warp][e] = __popc(peers);
    __syncthreads();
    int pos = -1;
    if (e >= 0) {
      pos = s_next[e] + rank;
      for (int w = 0; w < warp; ++w) pos += s_wcnt[w][e];
      sorted_entry[pos] = (int32_t)j;
    }
    s_pos[threadIdx.x] = pos;
    s_tok[threadIdx.x] = j / k;
    __syncthreads();
    for (int e2 = threadIdx.x; e2 < E; e2 += blockDim.x) {
      int add = 0;
      for (int w = 0; w < kWarps; ++w) add += s_wcnt[w][e2];
      s_next[e2] += add;
    }
    // each warp copies the rows of its 32 entries, 16 bytes per lane, eight
    // rows (sixteen loads per lane) in flight at a time
    for (int c0 = 0; c0 < chunks16; c0 += 64) {
      for (int q0 = 0; q0 < 32; q0 += 8) {
        uint4 v[8][2];
        int pq[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int t = warp * 32 + q0 + u;
          pq[u] = s_pos[t];
          const uint4* src = reinterpret_cast<const uint4*>(x + s_tok[t] * x_pitch);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = c0 + lane + 32 * h;
            if (pq[u] >= 0 && c < chunks16) v[u][h] = __ldg(src + c);
          }
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          uint4* dst = reinterpret_cast<uint4*>(packed + (int64_t)pq[u] * row_bytes);
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int c = c0 + lane + 32 * h;
            if (pq[u] >= 0 && c < chunks16) dst[c] = v[u][h];
          }
        }
      }
    }
  }
}

// out[t] = y[t*k] + y[t*k+1] + ... (each sum rounded to T), 8 values per lane
// step; entries with an invalid expert id add nothing.  One warp per token.
template <typename T, typename IdxT>
__global__ void __launch_bounds__(256) combine_kernel(const T* __restrict__ y, const IdxT* __restrict__ idx, int64_t Tn,
                                                      int k, int E, int D, T* __restrict__ out, int64_t ldo) {
  const int64_t t = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= Tn) return;
  const int lane = threadIdx.x & 31;
  if (k == 2 && D == 512) {
    // the SMoE's top-2 at d_model 512: both routes' ids, then all four 16-byte
    // row pieces of the lane requested before any arithmetic
    const int64_t v0 = (int64_t)idx[2 * t], v1 = (int64_t)idx[2 * t + 1];
    const bool ok0 = v0 >= 0 && v0 < E, ok1 = v1 >= 0 && v1 < E;
    const uint4* y0 = reinterpret_cast<const uint4*>(y + (2 * t) * (int64_t)512) + lane;
    const uint4* y1 = reinterpret_cast<const uint4*>(y + (2 * t + 1) * (int64_t)512) + lane;
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    uint4 w[2][2];
    w[0][0] = ok0 ? __ldg(y0) : zero;
    w[0][1] = ok0 ? __ldg(y0 + 32) : zero;
    w[1][0] = ok1 ? __ldg(y1) : zero;
    w[1][1] = ok1 ? __ldg(y1 + 32) : zero;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        if (!(s == 0 ? ok0 : ok1)) continue;
        const T* hv = reinterpret_cast<const T*>(&w[s][h]);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = (float)T(acc[i] + (float)hv[i]);
      }
      uint4 o;
      T* oh = reinterpret_cast<T*>(&o);
#pragma unroll
      for (int i = 0; i < 8; ++i) oh[i] = T(acc[i]);
      *reinterpret_cast<uint4*>(out + t * ldo + 8 * lane + 256 * h) = o;
    }
    return;
  }
  for (int c = lane * 8; c < D; c += 32 * 8) {
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    for (int s = 0; s < k; ++s) {
      const int64_t v = (int64_t)idx[t * k + s];
      if (v < 0 || v >= E) continue;
      const uint4 w = __ldg(reinterpret_cast<const uint4*>(y + (t * k + s) * (int64_t)D + c));
      const T* h = reinterpret_cast<const T*>(&w);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float sum = acc[i] + (float)h[i];
        acc[i] = (float)T(sum);
      }
    }
    uint4 o;
    T* oh = reinterpret_cast<T*>(&o);
#pragma unroll
    for (int i = 0; i < 8; ++i) oh[i] = T(acc[i]);
    *reinterpret_cast<uint4*>(out + t * ldo + c) = o;
  }
}

// ------------------------------------------------------------ grouped GEMM
using tc::BK;

constexpr int MMA_KB = 32;      // K bytes per tcgen05.mma kind::f16 (16 elements)
constexpr int kPairRows = 256;  // rows of a tile (128 per CTA of the pair)
constexpr int kTileCols = 256;  // columns of a tile
// a TMA warp, an MMA warp and eight epilogue warps (two per TMEM lane quarter,
// one per half of the tile's columns)
constexpr int kMoeEpiWarps = 8;
constexpr int kMoeThreads = 64 + 32 * kMoeEpiWarps;
using PairCfg = tc::pair::Cfg<256>;  // 6-stage ring of 16 KB of A + 16 KB of B per CTA, 512 TMEM columns

// instruction descriptor: D = F32, A/B = BF16 or F16, both K-major, M = 256 (the pair), N = 256
template <typename T>
struct F16KindPair;
template <>
struct F16KindPair<__nv_bfloat16> {
  static constexpr uint32_t idesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kTileCols >> 3) << 17) |
                                    ((uint32_t)(kPairRows >> 4) << 24);
};
template <>
struct F16KindPair<__half> {
  static constexpr uint32_t idesc = (1u << 4) | ((uint32_t)(kTileCols >> 3) << 17) | ((uint32_t)(kPairRows >> 4) << 24);
};

template <typename T>
__device__ __forceinline__ void umma_f16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8, %9, %10, %11, %12}, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(F16KindPair<T>::idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u), "r"(0u),
      "r"(0u), "r"(0u), "r"(0u));
}

struct MoeGemmParams {
  const int32_t* offsets;      // [E+1] row offset of each expert's segment of A
  const int32_t* sorted_entry; // [R] routed entry of each row of A (epilogue 2)
  const void* score;           // [R] gate score of each routed entry (epilogue 2), T
  const void* bias;            // [E * N] in T, or null
  void* out;                   // epilogue 1: hidden [R, ldo]; epilogue 2: y [R, ldo] by entry
  int64_t ldo;
  int E;
  int N;  // output columns per expert
  int K;  // reduction length
};

template <typename T>
__device__ __forceinline__ float round_to(float v) {
  return (float)T(v);
}

// Epilogue of one finished 128-row x 256-column accumulator (this CTA's rows
// m0 .. m0+127 of expert e, columns n0 ..): a warp with TMEM lane quarter
// `quarter` reads lanes 32*quarter.. of the 32-column chunks c_begin ..
// c_end-1 of the accumulator at TMEM column t_acc, rounds as the reference's
// torch ops do and stores the live rows (below m_end).
template <int EPI, typename T>
__device__ __forceinline__ void moe_epilogue_tile(const MoeGemmParams& p, int e, int m0, int m_end, int n0,
                                                  int quarter, int lane, uint32_t t_acc, int c_begin, int c_end) {
  const T* bias = reinterpret_cast<const T*>(p.bias);
  const int row = m0 + quarter * 32 + lane;
  const bool live = row < m_end;
  int64_t orow = row;
  float w = 0.0f;
  if (EPI == 2 && live) {
    const int32_t entry = p.sorted_entry[row];
    orow = entry;
    w = (float)reinterpret_cast<const T*>(p.score)[entry];
  }
#pragma unroll 1
  for (int c = c_begin; c < c_end; ++c) {
    const int col0 = n0 + c * 32;
    if (col0 >= p.N) break;  // warp-uniform
    // the chunk's 32 bias values (four 16-byte loads when aligned), requested
    // before the TMEM load so that the two latencies overlap
    T bv[32];
    if (bias != nullptr) {
      const T* bp = bias + (int64_t)e * p.N + col0;
      if ((reinterpret_cast<uintptr_t>(bp) & 15) == 0 && col0 + 32 <= p.N) {
#pragma unroll
        for (int q = 0; q < 4; ++q) *reinterpret_cast<uint4*>(bv + 8 * q) = __ldg(reinterpret_cast<const uint4*>(bp) + q);
      } else {
#pragma unroll
        for (int q = 0; q < 32; ++q) bv[q] = col0 + q < p.N ? bp[q] : T(0.0f);
      }
    }
    uint32_t r[32];
    tc::tmem_ld32(t_acc + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(c * 32), r);
    if (!live) continue;
    uint32_t packed[16];
    if constexpr (std::is_same<T, __nv_bfloat16>::value) {
      if (bias != nullptr) {
        // bf16 with bias, pairs of columns: the bmm result rounded (one
        // cvt for both), widened, + bias as the bf16 operand of a mixed
        // fp32 add, then (1) relu before the rounding -- exact here: a sum
        // of two bf16 values is 0, -0 or at least 2^-133 in magnitude, so
        // it is negative exactly when its rounding is -- or (2) rounded,
        // widened, times the score and rounded; one cvt packs each pair
        const uint32_t* bw = reinterpret_cast<const uint32_t*>(bv);
        const F2 w2 = f2(w, w);
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const uint32_t p1 = pack_bf16x2(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
          float lo = add_lo(bf16_lo(p1), bw[j]), hi = add_hi(bf16_hi(p1), bw[j]);
          if (EPI == 1) {
            lo = lo < 0.0f ? 0.0f : lo;
            hi = hi < 0.0f ? 0.0f : hi;
            packed[j] = pack_bf16x2(lo, hi);
          } else {
            const uint32_t p2 = pack_bf16x2(lo, hi);
            const float2 v = un(mul2v(f2(bf16_lo(p2), bf16_hi(p2)), w2));
            packed[j] = pack_bf16x2(v.x, v.y);
          }
        }
        T* dst = reinterpret_cast<T*>(p.out) + orow * p.ldo + col0;
        stg_v8(dst, packed);
        stg_v8(dst + 16, packed + 8);
        continue;
      }
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      float v2[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v = round_to<T>(__uint_as_float(r[2 * j + h]));
        if (bias != nullptr) v = round_to<T>(__fadd_rn(v, (float)bv[2 * j + h]));
        if (EPI == 1) {
          v = v < 0.0f ? 0.0f : v;
        } else {
          v = round_to<T>(__fmul_rn(v, w));
        }
        v2[h] = v;
      }
      T lo = T(v2[0]), hi = T(v2[1]);
      packed[j] = (uint32_t)(*reinterpret_cast<uint16_t*>(&lo)) | ((uint32_t)(*reinterpret_cast<uint16_t*>(&hi)) << 16);
    }
    T* dst = reinterpret_cast<T*>(p.out) + orow * p.ldo + col0;
    stg_v8(dst, packed);
    stg_v8(dst + 16, packed + 8);
  }
}

// The grouped GEMM on CTA pairs: a cluster of two CTAs computes each 256 x 256
// tile (expert, 256-row block, 256-column block) with
// tcgen05.mma.cta_group::2 issued by the leader; each CTA TMA-loads its own 128
// rows of A and 128 rows of B per stage (no multicast) and signals the leader's
// full barrier, and the leader's commits arrive on both CTAs' barriers.  Per SM
// a stage carries 16 KB of A and 16 KB of B for the MMA work that costs a
// one-SM 128 x 256 tile 16 KB of A and 32 KB of B.  A persistent pair walks the
// tiles of all experts, reading the segment offsets on the device; rows of a
// block past its expert's segment are computed and discarded.  Each CTA's
// eight epilogue warps round and store its 128 rows, two warps per TMEM lane
// quarter (one per half of the columns): at d_model 512 a tile's main loop is
// only 8 (FC1) or 16 (FC2) ring stages, and four epilogue warps fell behind
// it.  The epilogue warps of both CTAs release an accumulator on the leader's
// barrier.
template <int EPI, typename T>
__global__ void __launch_bounds__(kMoeThreads, 1)
    moe_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                         const __grid_constant__ MoeGemmParams p) {
  namespace pr = tc::pair;
  constexpr int kStages = PairCfg::STAGES;
  constexpr int kStageBytes = PairCfg::STAGE_BYTES;
  constexpr int kABytes = pr::A_BYTES;
  constexpr int kBBytes = PairCfg::B_BYTES;
  constexpr int kTmemCols = PairCfg::TMEM_COLS;
  constexpr int kElt = (int)sizeof(T);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
  uint8_t* sA = smem;
  uint8_t* sB = smem + kStages * kABytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;                 // [kStages]  leader: TMA bytes of both CTAs -> MMA
  uint64_t* empty = bars + kStages;      // [kStages]  both: MMA done with the slot -> TMA
  uint64_t* tfull = bars + 2 * kStages;  // [2]        both: accumulator ready -> epilogue
  uint64_t* tempty = tfull + 2;          // [2]        leader: both epilogues done -> MMA
  uint64_t* done = tempty + 2;           // [1]        leader: all MMAs complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  __shared__ int s_off[kMaxExperts + 1];
  __shared__ int s_mt[kMaxExperts + 1];  // prefix of 256-row blocks per expert

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = pr::cluster_rank();
  const bool leader = rank == 0;
  const int E = p.E;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&tfull[b]), 1);
      mbar_init(smem_u32(&tempty[b]), 2 * kMoeEpiWarps);  // one arrival per epilogue warp of both CTAs
    }
    mbar_init(smem_u32(done), 1);
    *abort_flag = 0;
    int mt = 0;
    for (int e = 0; e < E; ++e) {
      const int a = p.offsets[e], b = p.offsets[e + 1];
      s_off[e] = a;
      s_mt[e] = mt;
      mt += (b - a + kPairRows - 1) / kPairRows;
    }
    s_off[E] = p.offsets[E];
    s_mt[E] = mt;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 0 && lane == 0) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmA)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmB)) : "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tc::tc_fence_before();
  __syncthreads();
  pr::cluster_sync_all();  // both CTAs' barriers are initialised before any remote arrival
  tc::tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int n_tiles = (p.N + kTileCols - 1) / kTileCols;
  const int64_t num_tiles = (int64_t)s_mt[E] * n_tiles;
  const int kblocks = (int)(((int64_t)p.K * kElt + BK - 1) / BK);
  const int64_t pair_id = blockIdx.x >> 1;
  const int64_t num_pairs = gridDim.x >> 1;
  // tile -> (expert, first row of the tile, end of the expert's rows, first
  // column); n is the fastest index so pairs running side by side share their
  // A rows in L2
  auto locate = [&](int64_t tile, int& e, int& m0, int& m_end, int& n0) {
    const int mg = (int)(tile / n_tiles);
    n0 = (int)(tile % n_tiles) * kTileCols;
    e = 0;
    while (e + 1 < E && s_mt[e + 1] <= mg) ++e;
    m0 = s_off[e] + (mg - s_mt[e]) * kPairRows;
    m_end = s_off[e + 1];
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- producer
      const uint64_t pol_a = tc::policy_evict_first(), pol_b = tc::policy_evict_last();
      int stage = 0;
      uint32_t phase = 0, issued = 0, issued_phase = 0;
      bool ok = true;
      for (int64_t tile = pair_id; tile < num_tiles && ok; tile += num_pairs) {
        int e, m0, m_end, n0;
        locate(tile, e, m0, m_end, n0);
        const int arow = m0 + (int)rank * 128;
        const int brow = e * p.N + n0 + (int)rank * 128;
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&empty[stage]), phase ^ 1, kWaitTimeoutProducer, abort_flag)) {
            ok = false;
            break;
          }
          const uint32_t fb_local = smem_u32(&full[stage]);
          if (leader) mbar_arrive_expect_tx(fb_local, 2 * kStageBytes);
          const uint32_t fb = pr::map_rank(fb_local, 0);
          pr::tma_load_2d_pair(smem_u32(sA + stage * kABytes), &tmA, kb * (BK / kElt), arow, fb, pol_a);
          pr::tma_load_2d_pair(smem_u32(sB + stage * kBBytes), &tmB, kb * (BK / kElt), brow, fb, pol_b);
          issued |= 1u << stage;
          issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (leader) {
        // the leader's full barriers count both CTAs' bytes: drain them before exit
        for (int s = 0; s < kStages; ++s)
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
        tc::tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * kTileCols);
        for (int kb = 0; kb < kblocks; ++kb) {
          if (!mbar_wait_bounded(smem_u32(&full[stage]), phase, kWaitTimeoutMma, abort_flag)) {
            ok = false;
            break;
          }
          tc::tc_fence_after();
          const uint64_t adesc = tc::sw128_desc(smem_u32(sA + stage * kABytes));
          const uint64_t bdesc = tc::sw128_desc(smem_u32(sB + stage * kBBytes));
#pragma unroll
          for (int s = 0; s < BK / MMA_KB; ++s)
            umma_f16_pair<T>(d_tmem, adesc + (uint64_t)(s * MMA_KB / 16), bdesc + (uint64_t)(s * MMA_KB / 16),
                             (kb > 0 || s > 0) ? 1u : 0u);
          pr::umma_commit_both(smem_u32(&empty[stage]));
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        pr::umma_commit_both(smem_u32(&tfull[acc]));
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
    const int quarter = warp & 3;  // the TMEM lanes this warp can read
    constexpr int kChunks = kTileCols / 32 / (kMoeEpiWarps / 4);  // 32-column chunks per epilogue warp
    const int c_begin = ((warp - 2) >> 2) * kChunks;
    const uint32_t tempty_leader0 = pr::map_rank(smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = pr::map_rank(smem_u32(&tempty[1]), 0);
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int64_t tile = pair_id; tile < num_tiles; tile += num_pairs) {
      int e, m0, m_end, n0;
      locate(tile, e, m0, m_end, n0);
      if (!mbar_wait_bounded(smem_u32(&tfull[acc]), acc_phase, kWaitTimeoutEpilogue, abort_flag)) break;
      tc::tc_fence_after();
      moe_epilogue_tile<EPI, T>(p, e, m0 + (int)rank * 128, m_end, n0, quarter, lane,
                                tmem_base + (uint32_t)(acc * kTileCols), c_begin, c_begin + kChunks);
      tc::tc_fence_before();
      __syncwarp();
      if (lane == 0) pr::mbar_arrive_remote(acc ? tempty_leader1 : tempty_leader0);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1;
    }
  }

  tc::tc_fence_before();
  __syncthreads();
  pr::cluster_sync_all();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc::tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}
static std::once_flag g_moe_attr_once[64];

struct Workspace {
  int32_t* chunk_hist;
  int32_t* offsets;
  int32_t* sorted_entry;
  uint8_t* rows;    // packed x rows, then the weighted expert outputs y (same bytes)
  uint8_t* hidden;  // [R, F]
  int64_t bytes;
};

static int64_t align256(int64_t v) { return (v + 255) & ~(int64_t)255; }

static Workspace layout(void* base, int64_t R, int E, int D, int F, int elt) {
  Workspace w{};
  const int64_t nchunks = (R + kRouteChunk - 1) / kRouteChunk;
  uint8_t* b = static_cast<uint8_t*>(base);
  int64_t o = 0;
  w.chunk_hist = reinterpret_cast<int32_t*>(b + o);
  o += align256(nchunks * E * 4);
  w.offsets = reinterpret_cast<int32_t*>(b + o);
  o += align256((E + 1) * 4);
  w.sorted_entry = reinterpret_cast<int32_t*>(b + o);
  o += align256(R * 4);
  w.rows = b + o;
  o += align256(R * (int64_t)D * elt);
  w.hidden = b + o;
  o += align256(R * (int64_t)F * elt);
  w.bytes = o;
  return w;
}

}  // namespace moe
}  // namespace rb

using namespace rb;

extern "C" int64_t rb_smoe_workspace_size(int64_t T, int k, int E, int D, int F, int x_dtype) {
  if (T < 0 || k <= 0 || E <= 0 || D <= 0 || F <= 0) return -1;
  const int elt = dtype_size(x_dtype);
  if (elt != 2) return -1;
  return moe::layout(nullptr, T * k, E, D, F, elt).bytes;
}

extern "C" int rb_smoe_experts(const void* x, int x_dtype, int64_t ldx, int64_t T, int D, const void* topk_idx,
                               int idx_dtype, const void* topk_score, int k, int E, const void* w1, const void* b1,
                               const void* w2, const void* b2, int F, void* workspace, int64_t workspace_bytes,
                               void* out, int64_t ldo, void* stream) {
  using namespace rb::moe;
  if (T < 0 || k <= 0 || E <= 0 || D <= 0 || F <= 0) return fail(RB_ERR_VALUE, "negative or empty SMoE shape");
  if (x_dtype != RB_BF16 && x_dtype != RB_F16) return fail(RB_ERR_UNSUPPORTED, "rb_smoe_experts takes bf16 or f16");
  if (idx_dtype != RB_I64 && idx_dtype != RB_I32) return fail(RB_ERR_VALUE, "topk_idx must be int64 or int32");
  if (E > kMaxExperts) return fail(RB_ERR_UNSUPPORTED, "more than %d experts", kMaxExperts);
  if (D % 64 != 0 || F % 64 != 0) return fail(RB_ERR_UNSUPPORTED, "d_model and dim_ff must be multiples of 64");
  if ((int64_t)E * F > 0x7fffffffLL || (int64_t)E * D > 0x7fffffffLL) return fail(RB_ERR_UNSUPPORTED, "expert weights too large");
  if (T * k > 0x7fffffffLL) return fail(RB_ERR_UNSUPPORTED, "more than 2^31-1 routed entries");
  if (ldx < D || ldo < D) return fail(RB_ERR_VALUE, "leading dimension smaller than the row");
  if (T == 0) return RB_OK;
  if (x == nullptr || topk_idx == nullptr || topk_score == nullptr || w1 == nullptr || w2 == nullptr ||
      out == nullptr || workspace == nullptr)
    return fail(RB_ERR_VALUE, "null operand");
  const int elt = 2;
  if (!aligned(x, 16) || !aligned(out, 32) || (ldx * elt) % 16 != 0 || (ldo * elt) % 32 != 0 || !aligned(w1, 16) ||
      !aligned(w2, 16) || !aligned(workspace, 256))
    return fail(RB_ERR_VALUE, "x/out/weights/workspace misaligned (16-byte rows, 32-byte output rows, 256-byte workspace)");
  const int64_t R = T * k;
  const Workspace ws = layout(workspace, R, E, D, F, elt);
  if (workspace_bytes < ws.bytes) return fail(RB_ERR_VALUE, "workspace of %lld bytes, %lld needed",
                                              (long long)workspace_bytes, (long long)ws.bytes);
  if (!device_is_sm100()) return fail(RB_ERR_DEVICE, "rb_smoe_experts needs an sm_100 (B200) device");
  cudaStream_t st = (cudaStream_t)stream;
  const int nchunks = (int)((R + kRouteChunk - 1) / kRouteChunk);
  if (idx_dtype == RB_I64) {
    route_count_kernel<int64_t><<<nchunks, kRouteThreads, 0, st>>>(static_cast<const int64_t*>(topk_idx), R, E,
                                                                   ws.chunk_hist);
    route_scatter_kernel<int64_t><<<nchunks, kRouteThreads, 0, st>>>(
        static_cast<const int64_t*>(topk_idx), R, k, E, nchunks, ws.chunk_hist, ws.offsets, ws.sorted_entry,
        static_cast<const uint8_t*>(x), ldx * elt, (int64_t)D * elt, ws.rows);
  } else {
    route_count_kernel<int32_t><<<nchunks, kRouteThreads, 0, st>>>(static_cast<const int32_t*>(topk_idx), R, E,
                                                                   ws.chunk_hist);
    route_scatter_kernel<int32_t><<<nchunks, kRouteThreads, 0, st>>>(
        static_cast<const int32_t*>(topk_idx), R, k, E, nchunks, ws.chunk_hist, ws.offsets, ws.sorted_entry,
        static_cast<const uint8_t*>(x), ldx * elt, (int64_t)D * elt, ws.rows);
  }
  int rc = check_cuda(cudaGetLastError(), "SMoE route launch");
  if (rc) return rc;

  const CUtensorMapDataType dt = x_dtype == RB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  // A in 128-row boxes, B in 128-row boxes: each CTA of a pair loads its half of a 256 x 256 tile
  CUtensorMap tA1, tB1, tA2, tB2;
  if ((rc = tc::make_tmap(&tA1, ws.rows, D, R, (int64_t)D * elt, tc::BK / elt, 128, dt))) return rc;
  if ((rc = tc::make_tmap(&tB1, w1, D, (int64_t)E * F, (int64_t)D * elt, tc::BK / elt, 128, dt))) return rc;
  if ((rc = tc::make_tmap(&tA2, ws.hidden, F, R, (int64_t)F * elt, tc::BK / elt, 128, dt))) return rc;
  if ((rc = tc::make_tmap(&tB2, w2, F, (int64_t)E * D, (int64_t)F * elt, tc::BK / elt, 128, dt))) return rc;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaError_t attr_err = cudaSuccess;
  std::call_once(g_moe_attr_once[dev & 63], [&] {
    const void* fns[4] = {(const void*)moe_gemm_pair_kernel<1, __nv_bfloat16>,
                          (const void*)moe_gemm_pair_kernel<2, __nv_bfloat16>,
                          (const void*)moe_gemm_pair_kernel<1, __half>, (const void*)moe_gemm_pair_kernel<2, __half>};
    for (const void* f : fns)
      if (attr_err == cudaSuccess)
        attr_err = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, PairCfg::SMEM_BYTES);
  });
  if (attr_err != cudaSuccess) return check_cuda(attr_err, "cudaFuncSetAttribute(moe_gemm_pair_kernel)");

  MoeGemmParams p1{};
  p1.offsets = ws.offsets;
  p1.bias = b1;
  p1.out = ws.hidden;
  p1.ldo = F;
  p1.E = E;
  p1.N = F;
  p1.K = D;
  MoeGemmParams p2 = p1;
  p2.sorted_entry = ws.sorted_entry;
  p2.score = topk_score;
  p2.bias = b2;
  p2.out = ws.rows;  // y by entry; the packed rows are dead once the first GEMM has run
  p2.ldo = D;
  p2.N = D;
  p2.K = F;
  // upper bound of the 256-row blocks over all experts: ceil(R / 256) + E
  const int64_t pblocks = (R + kPairRows - 1) / kPairRows + E;
  const int pairs_avail = sm_count() / 2;
  const int pairs1 = (int)std::min<int64_t>(pblocks * ((F + kTileCols - 1) / kTileCols), pairs_avail);
  const int pairs2 = (int)std::min<int64_t>(pblocks * ((D + kTileCols - 1) / kTileCols), pairs_avail);
  const unsigned cgrid = (unsigned)((T + 7) / 8);
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kMoeThreads);
  cfg.dynamicSmemBytes = PairCfg::SMEM_BYTES;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t le;
  cfg.gridDim = dim3(2 * pairs1);
  le = x_dtype == RB_BF16 ? cudaLaunchKernelEx(&cfg, moe_gemm_pair_kernel<1, __nv_bfloat16>, tA1, tB1, p1)
                          : cudaLaunchKernelEx(&cfg, moe_gemm_pair_kernel<1, __half>, tA1, tB1, p1);
  if (le != cudaSuccess) return check_cuda(le, "moe_gemm_pair_kernel<1> launch");
  cfg.gridDim = dim3(2 * pairs2);
  le = x_dtype == RB_BF16 ? cudaLaunchKernelEx(&cfg, moe_gemm_pair_kernel<2, __nv_bfloat16>, tA2, tB2, p2)
                          : cudaLaunchKernelEx(&cfg, moe_gemm_pair_kernel<2, __half>, tA2, tB2, p2);
  if (le != cudaSuccess) return check_cuda(le, "moe_gemm_pair_kernel<2> launch");
  if ((rc = check_cuda(cudaGetLastError(), "moe_gemm_pair_kernel launch"))) return rc;
  if (idx_dtype == RB_I64) {
    if (x_dtype == RB_BF16)
      combine_kernel<__nv_bfloat16, int64_t><<<cgrid, 256, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(ws.rows), static_cast<const int64_t*>(topk_idx), T, k, E, D,
          static_cast<__nv_bfloat16*>(out), ldo);
    else
      combine_kernel<__half, int64_t><<<cgrid, 256, 0, st>>>(reinterpret_cast<const __half*>(ws.rows),
                                                              static_cast<const int64_t*>(topk_idx), T, k, E, D,
                                                              static_cast<__half*>(out), ldo);
  } else {
    if (x_dtype == RB_BF16)
      combine_kernel<__nv_bfloat16, int32_t><<<cgrid, 256, 0, st>>>(
          reinterpret_cast<const __nv_bfloat16*>(ws.rows), static_cast<const int32_t*>(topk_idx), T, k, E, D,
          static_cast<__nv_bfloat16*>(out), ldo);
    else
      combine_kernel<__half, int32_t><<<cgrid, 256, 0, st>>>(reinterpret_cast<const __half*>(ws.rows),
                                                             static_cast<const int32_t*>(topk_idx), T, k, E, D,
                                                             static_cast<__half*>(out), ldo);
  }
  return check_cuda(cudaGetLastError(), "SMoE combine launch");
}
