// common.cuh -- shared helpers of the sm_100a RepEncoder library: dtype
// conversion, host-side error reporting, the device watchdog word and the
// bounded mbarrier wait used by every pipelined kernel.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/rep_b200.h"

namespace rb {

// ------------------------------------------------------------ host errors
void set_error(const char* fmt, ...);
int fail(int code, const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);
int sm_count();
bool device_is_sm100();

// First non-zero watchdog code of any kernel in this library (0 = healthy).
// Defined here: the library is built as one translation unit (rep_b200_all.cu).
__device__ int g_device_error = 0;

enum WatchdogCode : int {
  kWaitTimeoutProducer = 101,
  kWaitTimeoutMma = 102,
  kWaitTimeoutEpilogue = 103,
  kWaitTimeoutSelftest = 199,
};

// Default budget for one mbarrier wait inside a kernel: 2 s of wall time.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ void raise_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(bar), "r"(parity)
      : "memory");
  return done != 0;
}

// Wait for the phase with the given parity to complete, for at most
// budget_ns of wall time.  Returns false (and records `code`) on timeout, or
// immediately when *abort is set by another role of the same CTA.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity, int code,
                                                  volatile int* abort_flag,
                                                  uint64_t budget_ns = kWaitBudgetNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (abort_flag != nullptr && *abort_flag) return false;
    if (global_ns() - t0 > budget_ns) {
      raise_device_error(code);
      if (abort_flag != nullptr) *abort_flag = 1;
      return false;
    }
  }
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(bar)
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(bar),
      "r"(bytes)
      : "memory");
}

// ----------------------------------------------------------------- dtypes
__device__ __forceinline__ float load_as_f32(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case RB_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case RB_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}

// ------------------------------------------------------------ f32x2 math
// Blackwell packed fp32: one instruction performs two IEEE round-to-nearest
// operations.  Lanes of a pair are independent, so results equal the scalar ops.
// A multiply whose result feeds an add must use mul2v / add2v: a build of this
// library turned a plain asm multiply-then-add into one rounding instead of
// two.  The volatile forms keep both roundings; they are not used everywhere
// because they also stop the compiler from scheduling around them (K1 ran 19 %
// slower with every helper volatile, with bit-identical results).
struct F2 {
  unsigned long long r;
};
__device__ __forceinline__ F2 f2(float lo, float hi) {
  F2 v;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v.r) : "f"(lo), "f"(hi));
  return v;
}
__device__ __forceinline__ float2 un(F2 v) {
  float2 o;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(o.x), "=f"(o.y) : "l"(v.r));
  return o;
}
__device__ __forceinline__ F2 add2(F2 a, F2 b) {
  F2 d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d.r) : "l"(a.r), "l"(b.r));
  return d;
}
__device__ __forceinline__ F2 sub2(F2 a, F2 b) {
  F2 d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d.r) : "l"(a.r), "l"(b.r));
  return d;
}
__device__ __forceinline__ F2 mul2(F2 a, F2 b) {
  F2 d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d.r) : "l"(a.r), "l"(b.r));
  return d;
}
__device__ __forceinline__ F2 fma2(F2 a, F2 b, F2 c) {
  F2 d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d.r) : "l"(a.r), "l"(b.r), "l"(c.r));
  return d;
}
__device__ __forceinline__ F2 mul2v(F2 a, F2 b) {
  F2 d;
  asm volatile("mul.rn.f32x2 %0, %1, %2;" : "=l"(d.r) : "l"(a.r), "l"(b.r));
  return d;
}
__device__ __forceinline__ F2 add2v(F2 a, F2 b) {
  F2 d;
  asm volatile("add.rn.f32x2 %0, %1, %2;" : "=l"(d.r) : "l"(a.r), "l"(b.r));
  return d;
}
__device__ __forceinline__ F2 addrz2(F2 a, F2 b) {
  F2 d;
  asm("add.rz.f32x2 %0, %1, %2;" : "=l"(d.r) : "l"(a.r), "l"(b.r));
  return d;
}
// 32 bytes at p (32-byte aligned) in one 256-bit store: a lane fills a whole
// 32-byte sector with one instruction
__device__ __forceinline__ void stg_v8(void* p, const uint32_t* w) {
  asm volatile("st.global.v8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"l"(p), "r"(w[0]), "r"(w[1]),
               "r"(w[2]), "r"(w[3]), "r"(w[4]), "r"(w[5]), "r"(w[6]), "r"(w[7])
               : "memory");
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // RNE, lo in the low half
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float round_bf16(float v) {
  return __bfloat162float(__float2bfloat16_rn(v));
}

__device__ __forceinline__ uint32_t pack_i8x4(int a, int b, int c, int d) {
  return (uint32_t)(a & 0xff) | ((uint32_t)(b & 0xff) << 8) | ((uint32_t)(c & 0xff) << 16) |
         ((uint32_t)(d & 0xff) << 24);
}

__host__ __device__ inline int dtype_size(int dt) {
  switch (dt) {
    case RB_F32: case RB_I32: return 4;
    case RB_BF16: case RB_F16: return 2;
    case RB_I8: return 1;
    default: return 0;
  }
}

__host__ __device__ inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

}  // namespace rb
