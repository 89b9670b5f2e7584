// update_kernels.cu -- elementwise kernels of the PPO update's fp32-accurate split products.
//
// The reference's update (R/cuda_fdm/ppo_gpu.py:2020-2144) multiplies in fp32 with cuBLAS
// SGEMM.  Here each fp32 operand is carried as three bf16 terms [mid | lo | hi] so a product
// runs on the bf16 tensor cores with fp32 accumulation (the GEMMs themselves are cuBLAS calls
// made by the host).  The kernels below produce those terms where the data is already being
// touched:
//
//   k_split3          the split of an fp32 matrix (layer inputs, weights);
//   k_bias_act_split  a layer's epilogue: h = act(y + bias) in place, plus the split of h that
//                     the next layer's products read;
//   k_act_grad_split  a layer's backward prologue: g_y = g_h * act'(h), its split, and per-block
//                     column sums of g_y (the bias gradient, reduced over blocks by the host in
//                     a fixed order).
//
// Every part of a split row is `cols` rounded up to 8 columns (16 bytes of bf16), the pad columns
// zero, so every part starts 16-byte aligned for the tensor-core GEMMs.
#include <cuda_bf16.h>
#include "common.cuh"

namespace f16 {
namespace upd {

constexpr int THREADS = 256;
constexpr int MAX_GRAD_COLS = 4 * THREADS;   // one column group of 4 per thread of a block

__host__ __device__ __forceinline__ int part_of(int cols) { return (cols + 7) & ~7; }

// hi = bf16(v), lo = bf16(v - hi), mid = bf16(v - hi - lo), round to nearest; both differences
// are exact in fp32 (each is v minus a prefix of v's significand), so mid + lo + hi carries all
// 24 significant bits of v.  Stored as the row's mid, lo and hi parts.
__device__ __forceinline__ void split_store(const float a[4], __nv_bfloat16* o, int part) {
  __nv_bfloat16 hi[4], lo[4], mi[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    hi[k] = __float2bfloat16_rn(a[k]);
    const float r1 = __fsub_rn(a[k], __bfloat162float(hi[k]));
    lo[k] = __float2bfloat16_rn(r1);
    mi[k] = __float2bfloat16_rn(__fsub_rn(r1, __bfloat162float(lo[k])));
  }
  *reinterpret_cast<uint2*>(o) = *reinterpret_cast<const uint2*>(mi);
  *reinterpret_cast<uint2*>(o + part) = *reinterpret_cast<const uint2*>(lo);
  *reinterpret_cast<uint2*>(o + 2 * part) = *reinterpret_cast<const uint2*>(hi);
}

__device__ __forceinline__ void zero_store(__nv_bfloat16* o, int part) {
  const uint2 z = make_uint2(0u, 0u);
  *reinterpret_cast<uint2*>(o) = z;
  *reinterpret_cast<uint2*>(o + part) = z;
  *reinterpret_cast<uint2*>(o + 2 * part) = z;
}

// torch.relu (clamp_min(v, 0), NaN kept) / torch.tanh / identity.
__device__ __forceinline__ float act_fwd(float v, int act) {
  if (act == F16_ACT_RELU) return (v > 0.0f || v != v) ? v : 0.0f;
  if (act == F16_ACT_TANH) return tanhf(v);
  return v;
}

// torch's threshold_backward(g, h, 0) (h <= 0 -> 0, else g) / tanh_backward (g (1 - h h), the
// difference formed with one rounding as a fused multiply-add: exact cancellation near |h| = 1).
__device__ __forceinline__ float act_bwd(float g, float h, int act) {
  if (act == F16_ACT_RELU) return h <= 0.0f ? 0.0f : g;
  if (act == F16_ACT_TANH) return __fmul_rn(g, __fmaf_rn(-h, h, 1.0f));
  return g;
}

// One thread per 4 consecutive columns of a row part (16-byte load; 8-byte stores of each term).
__global__ void __launch_bounds__(THREADS) k_split3(const float* __restrict__ x, int64_t rows, int cols, int64_t ldx,
                                                    __nv_bfloat16* __restrict__ out, int64_t ldo) {
  const int part = part_of(cols);
  const int g = part >> 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * g) return;
  const int64_t r = i / g;
  const int c = (int)(i % g) * 4;
  __nv_bfloat16* o = out + r * ldo + c;
  if (c >= cols) {
    zero_store(o, part);
    return;
  }
  const float4 v = *reinterpret_cast<const float4*>(x + r * ldx + c);
  const float a[4] = {v.x, v.y, v.z, v.w};
  split_store(a, o, part);
}

// h = act(y + bias) written over y; with hs, also the split of h.  Same thread map as k_split3
// (the pad groups exist only when hs is written).
__global__ void __launch_bounds__(THREADS) k_bias_act_split(float* __restrict__ y, int64_t rows, int cols, int64_t ldy,
                                                            const float* __restrict__ bias, int act,
                                                            __nv_bfloat16* __restrict__ hs, int64_t ldhs) {
  const int part = hs ? part_of(cols) : cols;
  const int g = part >> 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * g) return;
  const int64_t r = i / g;
  const int c = (int)(i % g) * 4;
  if (c >= cols) {
    zero_store(hs + r * ldhs + c, part);
    return;
  }
  float4* yp = reinterpret_cast<float4*>(y + r * ldy + c);
  const float4 v = *yp;
  const float4 b = *reinterpret_cast<const float4*>(bias + c);
  const float a[4] = {act_fwd(__fadd_rn(v.x, b.x), act), act_fwd(__fadd_rn(v.y, b.y), act),
                      act_fwd(__fadd_rn(v.z, b.z), act), act_fwd(__fadd_rn(v.w, b.w), act)};
  *yp = make_float4(a[0], a[1], a[2], a[3]);
  if (hs) split_store(a, hs + r * ldhs + c, part);
}

// g_y = act'(g_h, h), its split, and the column sums of g_y over the block's rows.  A block is
// RS row slots x G column groups of 4 (G = part / 4 <= THREADS, RS = THREADS / G); block b owns
// rows [b rpb, (b + 1) rpb), slot s walks rows s, s + RS, ...; each thread sums its column group
// in row order and the slots are added in slot order, so the partial sums are deterministic.
__global__ void __launch_bounds__(THREADS) k_act_grad_split(const float* __restrict__ gh, int64_t ldg,
                                                            const float* __restrict__ h, int64_t ldh, int64_t rows,
                                                            int cols, int act, __nv_bfloat16* __restrict__ gys,
                                                            int64_t ldgs, float* __restrict__ col_part, int64_t rpb) {
  __shared__ float4 red[THREADS];
  const int part = part_of(cols);
  const int G = part >> 2;
  const int RS = THREADS / G;
  const int tid = threadIdx.x;
  const int slot = tid / G;
  const int c = (tid % G) * 4;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (slot < RS) {
    const int64_t r0 = (int64_t)blockIdx.x * rpb;
    const int64_t r1 = r0 + rpb < rows ? r0 + rpb : rows;
    for (int64_t r = r0 + slot; r < r1; r += RS) {
      __nv_bfloat16* o = gys + r * ldgs + c;
      if (c >= cols) {
        zero_store(o, part);
        continue;
      }
      const float4 gv = *reinterpret_cast<const float4*>(gh + r * ldg + c);
      const float4 hv = act == F16_ACT_NONE ? gv : *reinterpret_cast<const float4*>(h + r * ldh + c);
      const float a[4] = {act_bwd(gv.x, hv.x, act), act_bwd(gv.y, hv.y, act), act_bwd(gv.z, hv.z, act),
                          act_bwd(gv.w, hv.w, act)};
      acc.x = __fadd_rn(acc.x, a[0]);
      acc.y = __fadd_rn(acc.y, a[1]);
      acc.z = __fadd_rn(acc.z, a[2]);
      acc.w = __fadd_rn(acc.w, a[3]);
      split_store(a, o, part);
    }
  }
  red[tid] = acc;
  __syncthreads();
  if (tid < G && c < cols) {
    float4 s = red[tid];
    for (int j = 1; j < RS; j++) {
      const float4 t = red[j * G + tid];
      s.x = __fadd_rn(s.x, t.x);
      s.y = __fadd_rn(s.y, t.y);
      s.z = __fadd_rn(s.z, t.z);
      s.w = __fadd_rn(s.w, t.w);
    }
    *reinterpret_cast<float4*>(col_part + (int64_t)blockIdx.x * cols + c) = s;
  }
}

inline unsigned grid_for(int64_t n) { return (unsigned)((n + THREADS - 1) / THREADS); }

}  // namespace upd
}  // namespace f16

using namespace f16;

extern "C" int f16_split3_bf16(const float* x, int64_t rows, int cols, int64_t ldx, void* out, int64_t ldo,
                               f16_stream_t stream) {
  if (!x || !out || rows <= 0 || cols <= 0 || cols % 4 || ldx < cols || ldo < 3 * (int64_t)upd::part_of(cols))
    return F16_ERR_ARG;
  if (!aligned(x, 16) || ldx % 4 || !aligned(out, 8) || ldo % 4) return F16_ERR_ALIGN;
  const int64_t n = rows * (upd::part_of(cols) / 4);
  upd::k_split3<<<upd::grid_for(n), upd::THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, rows, cols, ldx, reinterpret_cast<__nv_bfloat16*>(out), ldo);
  return launch_status();
}

extern "C" int f16_bias_act_split(float* y, int64_t rows, int cols, int64_t ldy, const float* bias, int act,
                                  void* hs, int64_t ldhs, f16_stream_t stream) {
  if (!y || !bias || rows <= 0 || cols <= 0 || cols % 4 || ldy < cols || act < F16_ACT_NONE || act > F16_ACT_TANH)
    return F16_ERR_ARG;
  if (hs && ldhs < 3 * (int64_t)upd::part_of(cols)) return F16_ERR_ARG;
  if (!aligned(y, 16) || ldy % 4 || !aligned(bias, 16) || (hs && (!aligned(hs, 8) || ldhs % 4))) return F16_ERR_ALIGN;
  const int64_t n = rows * ((hs ? upd::part_of(cols) : cols) / 4);
  upd::k_bias_act_split<<<upd::grid_for(n), upd::THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      y, rows, cols, ldy, bias, act, reinterpret_cast<__nv_bfloat16*>(hs), ldhs);
  return launch_status();
}

extern "C" int f16_act_grad_split(const float* gh, int64_t ldg, const float* h, int64_t ldh, int64_t rows, int cols,
                                  int act, void* gys, int64_t ldgs, float* col_part, int nblk, f16_stream_t stream) {
  if (!gh || !gys || !col_part || rows <= 0 || cols <= 0 || cols % 4 || cols > upd::MAX_GRAD_COLS || ldg < cols ||
      ldgs < 3 * (int64_t)upd::part_of(cols) || nblk <= 0 || act < F16_ACT_NONE || act > F16_ACT_TANH)
    return F16_ERR_ARG;
  if (act != F16_ACT_NONE && (!h || ldh < cols)) return F16_ERR_ARG;
  if (!aligned(gh, 16) || ldg % 4 || !aligned(gys, 8) || ldgs % 4 || !aligned(col_part, 16) ||
      (act != F16_ACT_NONE && (!aligned(h, 16) || ldh % 4)))
    return F16_ERR_ALIGN;
  const int64_t rpb = (rows + nblk - 1) / nblk;
  upd::k_act_grad_split<<<(unsigned)nblk, upd::THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      gh, ldg, h, ldh, rows, cols, act, reinterpret_cast<__nv_bfloat16*>(gys), ldgs, col_part, rpb);
  return launch_status();
}
