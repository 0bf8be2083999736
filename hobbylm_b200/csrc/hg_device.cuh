// Device-side building blocks shared by the decode and prefill kernels.
//
// Q8 "lane-chunked" row layout. hobby-rs keeps a Q8 row as nb blocks of 32 int8 (quant.rs:69-75)
// and its AVX2 dot (quant.rs:44-67) gives lane l (0..7) of block b the four bytes 4l..4l+3. On the
// GPU one thread owns one (row, lane) and walks the blocks in order, so a row is stored with each
// lane's words of four consecutive blocks adjacent:
//   full chunk c (blocks 4c..4c+3):  byte c*128 + l*16 + (b%4)*4 + j   (j = byte within the word)
//   tail block b >= 4*(nb/4):        byte (nb/4)*128 + (b - 4*(nb/4))*32 + l*4 + j
// so one 16-byte load gives a lane its words for 4 blocks and 8 lanes read 128 contiguous bytes.
// Scales are f32 [row][ss] with ss = nb rounded up to a multiple of 4 (16-byte aligned rows).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

#include "../../include/hobbygpu.h"

namespace hg {

constexpr int QK = 32;

__host__ __device__ inline int q8_ss(int nb) { return (nb + 3) & ~3; }

// Byte offset of element k (0..cols-1) of a row in the lane-chunked layout.
__host__ __device__ inline int q8_pos(int k, int nb) {
  int b = k >> 5, j = k & 31, l = j >> 2, bj = j & 3;
  int nc = nb >> 2;
  if (b < nc * 4) return (b >> 2) * 128 + l * 16 + (b & 3) * 4 + bj;
  return nc * 128 + (b - nc * 4) * 32 + l * 4 + bj;
}

// ---- exact arithmetic helpers (no contraction: the build uses --fmad=false) ----
__device__ __forceinline__ float fmul(float a, float b) { return __fmul_rn(a, b); }
__device__ __forceinline__ float fadd(float a, float b) { return __fadd_rn(a, b); }

// Programmatic dependent launch. A kernel launched with programmatic serialization may start while
// the previous kernel on the stream is still running. pdl_wait() returns once that kernel has
// completed and its writes are visible; every decode kernel calls it before reading anything the
// previous kernel wrote, and calls pdl_trigger() after it, so a kernel starts at most one kernel
// ahead: anything written two or more kernels earlier may be read before pdl_wait(). Without the
// launch attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// f32 exp pinned to the correctly rounded value: (float)exp((double)x). The CPU oracle uses the
// same definition, so sigmoid / silu / softmax weights match it bit for bit.
__device__ __forceinline__ float exp_cr(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float sigmoid_ref(float x) {  // ops.rs:75-77
  return __fdiv_rn(1.0f, fadd(1.0f, exp_cr(-x)));
}
__device__ __forceinline__ float silu_ref(float x) { return fmul(x, sigmoid_ref(x)); }  // ops.rs:80-82

// 8-lane horizontal sum of the lane group (lanes 8g..8g+7 of the warp) in the order
// ((l0+l4)+(l2+l6))+((l1+l5)+(l3+l7)) (quant.rs:61-65); every lane of the group gets the result.
__device__ __forceinline__ float hsum8_group(float v) {
  v = fadd(v, __shfl_xor_sync(0xffffffffu, v, 4));
  v = fadd(v, __shfl_xor_sync(0xffffffffu, v, 2));
  v = fadd(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Per-32 block quantization of one value per lane of a full warp (quant.rs:112-123):
// amax = max|x| over the block, d = amax/127, id = d>0 ? 1/d : 0, q = clamp(round(x*id), -127, 127).
// Returns q; *d_out gets d (same in every lane).
__device__ __forceinline__ int8_t quant_lane(float x, float* d_out) {
  float amax = warp_max(fabsf(x));
  float d = __fdiv_rn(amax, 127.0f);
  float id = d > 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  float r = roundf(fmul(x, id));
  r = fminf(fmaxf(r, -127.0f), 127.0f);
  *d_out = d;
  return (int8_t)(int)r;
}

// Quantize a row of n floats (n % 32 == 0) held in shared or global memory into lane-chunked int8
// (q_out, byte-addressed) and scales (d_out). Called by a whole block; warps take blocks.
__device__ inline void quant_row_block(const float* x, int n, int8_t* q_out, float* d_out) {
  int nb = n >> 5;
  int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int b = warp; b < nb; b += nw) {
    float d;
    int8_t q = quant_lane(x[b * 32 + lane], &d);
    q_out[q8_pos(b * 32 + lane, nb)] = q;
    if (lane == 0) d_out[b] = d;
  }
}

// Dot of one weight row with one quantized activation row for the calling (row, lane) thread:
// acc_l = fma(sw[b]*dx[b], float(p_l,b), acc_l) over blocks in order (quant.rs:50-59), with
// p_l,b = dp4a of the lane's word. Returns the lane accumulator (reduce with hsum8_group).
// wq/ws: this row's packed bytes and scales; aq/as: the activation row (shared memory).
template <int NB>
__device__ __forceinline__ float q8_lane_dot(const int8_t* __restrict__ wq, const float* __restrict__ ws,
                                             const int8_t* aq, const float* as, int lane) {
  constexpr int NC = NB / 4, NT = NB % 4;
  float acc = 0.0f;
#pragma unroll
  for (int c = 0; c < NC; c++) {
    int4 w = __ldg(reinterpret_cast<const int4*>(wq + c * 128 + lane * 16));
    float4 s = __ldg(reinterpret_cast<const float4*>(ws + c * 4));
    int4 a = *reinterpret_cast<const int4*>(aq + c * 128 + lane * 16);
    float4 d = *reinterpret_cast<const float4*>(as + c * 4);
    acc = __fmaf_rn(fmul(s.x, d.x), (float)__dp4a(w.x, a.x, 0), acc);
    acc = __fmaf_rn(fmul(s.y, d.y), (float)__dp4a(w.y, a.y, 0), acc);
    acc = __fmaf_rn(fmul(s.z, d.z), (float)__dp4a(w.z, a.z, 0), acc);
    acc = __fmaf_rn(fmul(s.w, d.w), (float)__dp4a(w.w, a.w, 0), acc);
  }
#pragma unroll
  for (int t = 0; t < NT; t++) {
    int w = __ldg(reinterpret_cast<const int*>(wq + NC * 128 + t * 32 + lane * 4));
    int a = *reinterpret_cast<const int*>(aq + NC * 128 + t * 32 + lane * 4);
    float s = __ldg(ws + NC * 4 + t);
    acc = __fmaf_rn(fmul(s, as[NC * 4 + t]), (float)__dp4a(w, a, 0), acc);
  }
  return acc;
}

// Runtime-nb fallback of q8_lane_dot (same arithmetic).
__device__ inline float q8_lane_dot_rt(const int8_t* __restrict__ wq, const float* __restrict__ ws,
                                       const int8_t* aq, const float* as, int lane, int nb) {
  int nc = nb >> 2, nt = nb & 3;
  float acc = 0.0f;
  for (int c = 0; c < nc; c++) {
    int4 w = __ldg(reinterpret_cast<const int4*>(wq + c * 128 + lane * 16));
    float4 s = __ldg(reinterpret_cast<const float4*>(ws + c * 4));
    int4 a = *reinterpret_cast<const int4*>(aq + c * 128 + lane * 16);
    float4 d = *reinterpret_cast<const float4*>(as + c * 4);
    acc = __fmaf_rn(fmul(s.x, d.x), (float)__dp4a(w.x, a.x, 0), acc);
    acc = __fmaf_rn(fmul(s.y, d.y), (float)__dp4a(w.y, a.y, 0), acc);
    acc = __fmaf_rn(fmul(s.z, d.z), (float)__dp4a(w.z, a.z, 0), acc);
    acc = __fmaf_rn(fmul(s.w, d.w), (float)__dp4a(w.w, a.w, 0), acc);
  }
  for (int t = 0; t < nt; t++) {
    int w = __ldg(reinterpret_cast<const int*>(wq + nc * 128 + t * 32 + lane * 4));
    int a = *reinterpret_cast<const int*>(aq + nc * 128 + t * 32 + lane * 4);
    float s = __ldg(ws + nc * 4 + t);
    acc = __fmaf_rn(fmul(s, as[nc * 4 + t]), (float)__dp4a(w, a, 0), acc);
  }
  return acc;
}

// ops::dot (ops.rs:7-36) of two n-float vectors (n % 32 == 0) by one warp: thread (m = lane/8,
// l = lane%8) is accumulator m's SIMD lane l, FMA-accumulating elements 32i + 8m + l in order i;
// then ((a0+a1)+(a2+a3)) per lane and the 8-lane tree. Returns the dot in every lane.
// The reduction of dot_ref_warp from each lane's accumulator: lane = 8m + l: combine m=0 with m=1
// (xor 8), m=2 with m=3 -> (a0+a1), (a2+a3); then xor 16; then the 8-lane tree.
__device__ __forceinline__ float dot_ref_warp_finish(float acc) {
  acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 8));
  acc = fadd(acc, __shfl_xor_sync(0xffffffffu, acc, 16));
  return hsum8_group(acc);
}
__device__ __forceinline__ float dot_ref_warp(const float* __restrict__ a, const float* __restrict__ b, int n) {
  int lane = threadIdx.x & 31;
  float acc = 0.0f;
  for (int i = 0; i < n; i += 32) acc = __fmaf_rn(a[i + lane], b[i + lane], acc);
  return dot_ref_warp_finish(acc);
}

// Orderable 32-bit key of a float (larger float -> larger key).
__device__ __forceinline__ uint32_t f2key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float key2f(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7fffffffu) : ~k);
}
// argmax key: high word = value key, low word = ~index so that the lowest index wins ties
// (sample.rs:53-64 keeps the first maximum).
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  return ((unsigned long long)f2key(v) << 32) | (unsigned long long)(0xffffffffu - idx);
}

}  // namespace hg
