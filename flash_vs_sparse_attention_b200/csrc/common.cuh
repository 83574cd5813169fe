// Shared helpers for the block-sparse attention kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "bsattn.h"  // from include/ (-I)

namespace bsa {

constexpr int kNumSMs = 148;  // B200

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// Pack two floats to bf16x2 with round-to-nearest-even (low half = a).
__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Pack two floats to fp16x2 with round-to-nearest-even (low half = a).
__device__ __forceinline__ uint32_t pack_f16x2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ float2 unpack_f16x2(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100: one instruction for two lanes of work).  Each
// half is rounded exactly as the scalar fmaf / fadd would round it.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " mov.b64 rc, {%6, %7};\n fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 r;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

__device__ __forceinline__ float fast_log2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^e for an integer e in [-126, 127], built from its exponent bits.
__device__ __forceinline__ float exp2i(int e) { return __int_as_float((e + 127) << 23); }

// max of three floats in one instruction (sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 1/ln(2): converts a natural-log-domain exponent to base 2.
constexpr float kLog2e = 1.4426950408889634f;

// Problem shape derived once on the host and passed by value to kernels.
struct Shape {
  int32_t units;       // batch * heads processed by this launch
  int32_t N;           // seq_len (of K and V; for decode, the cache capacity)
  int32_t D;           // head_dim
  int32_t bs;          // block_size
  int32_t nb;          // N / bs
  int32_t k;           // top_k
  int32_t causal;
  float scale;
  // Query rows and the valid key prefix.  The full forward has Nq = N,
  // q0 = 0, kv = N; decode has Nq new rows at positions q0 .. q0 + Nq - 1
  // against the first kv = q0 + Nq keys.  Only the CUDA-core kernels and the
  // decode selection read these; the tensor-core kernels run full forwards.
  int32_t Nq;          // query rows per unit (Q, O and idx unit stride)
  int32_t q0;          // position of query row 0
  int32_t kv;          // keys [0, kv) exist
  int32_t test_timeout;  // BSA_FLAG_TEST_TIMEOUT: the fine kernel's test hook
  // Per-head top_k (a per-head sparsity budget): device array of `heads`
  // budgets, or null (every row keeps k blocks).  Unit u of a launch is
  // head (unit0 + u) % heads; k is then the slot count of a row of idx.
  const int32_t* head_k;
  int32_t heads;
  int32_t unit0;
};

// Blocks a row of unit u keeps: its head's budget clamped to [1, k], or k.
__device__ __forceinline__ int unit_top_k(const Shape& s, int u) {
  if (s.head_k == nullptr) return s.k;
  const int kh = __ldg(s.head_k + (s.unit0 + u) % s.heads);
  return kh < 1 ? 1 : (kh > s.k ? s.k : kh);
}

}  // namespace bsa
