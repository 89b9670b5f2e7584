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
//                     a fixed order);
//   k_bias_act_value  the epilogue of a hidden layer followed by a width-1 Linear (the critic's
//                     value head), with the head's dot product; k_act_grad_split's value mode
//                     is its backward (the head's input gradient formed on the fly, the head's
//                     weight-gradient partial sums beside the bias partial sums);
//   k_cat_fwd/bwd     the categorical head on the actor's logits: summed log-prob of the taken
//                     actions and summed entropy per row, and their gradient.
//
// Every part of a split row is `cols` rounded up to 8 columns (16 bytes of bf16), the pad columns
// zero, so every part starts 16-byte aligned for the tensor-core GEMMs.  A split has three parts
// [mid | lo | hi] or six, [mid | lo | hi | lo | hi | hi]: the A operand of ONE GEMM over all six
// term products (against B = [hi; hi; mid; lo; lo; hi]), the hi*hi product last in K.
#include <cuda_bf16.h>
#include <cfloat>
#include "common.cuh"

namespace f16 {
namespace upd {

constexpr int THREADS = 256;
constexpr int MAX_GRAD_COLS = 4 * THREADS;   // one column group of 4 per thread of a block
constexpr int GRAD_UNROLL = 4;               // rows per pass of k_act_grad_split

__host__ __device__ __forceinline__ int part_of(int cols) { return (cols + 7) & ~7; }

// hi = bf16(v), lo = bf16(v - hi), mid = bf16(v - hi - lo), round to nearest; both differences
// are exact in fp32 (each is v minus a prefix of v's significand), so mid + lo + hi carries all
// 24 significant bits of v.  Stored as the row's mid, lo and hi parts, and with six parts also
// lo, hi, hi again (the A operand of a single GEMM over all six term products).
__device__ __forceinline__ void split_store(const float a[4], __nv_bfloat16* o, int part, bool six) {
  __nv_bfloat16 hi[4], lo[4], mi[4];
#pragma unroll
  for (int k = 0; k < 4; k++) {
    hi[k] = __float2bfloat16_rn(a[k]);
    const float r1 = __fsub_rn(a[k], __bfloat162float(hi[k]));
    lo[k] = __float2bfloat16_rn(r1);
    mi[k] = __float2bfloat16_rn(__fsub_rn(r1, __bfloat162float(lo[k])));
  }
  const uint2 m2 = *reinterpret_cast<const uint2*>(mi), l2 = *reinterpret_cast<const uint2*>(lo),
              h2 = *reinterpret_cast<const uint2*>(hi);
  *reinterpret_cast<uint2*>(o) = m2;
  *reinterpret_cast<uint2*>(o + part) = l2;
  *reinterpret_cast<uint2*>(o + 2 * part) = h2;
  if (six) {
    *reinterpret_cast<uint2*>(o + 3 * part) = l2;
    *reinterpret_cast<uint2*>(o + 4 * part) = h2;
    *reinterpret_cast<uint2*>(o + 5 * part) = h2;
  }
}

__device__ __forceinline__ void zero_store(__nv_bfloat16* o, int part, bool six) {
  const uint2 z = make_uint2(0u, 0u);
  const int n = six ? 6 : 3;
  for (int k = 0; k < n; k++) *reinterpret_cast<uint2*>(o + k * part) = z;
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
                                                    __nv_bfloat16* __restrict__ out, int64_t ldo, bool six) {
  const int part = part_of(cols);
  const int g = part >> 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * g) return;
  const int64_t r = i / g;
  const int c = (int)(i % g) * 4;
  __nv_bfloat16* o = out + r * ldo + c;
  if (c >= cols) {
    zero_store(o, part, six);
    return;
  }
  const float4 v = *reinterpret_cast<const float4*>(x + r * ldx + c);
  const float a[4] = {v.x, v.y, v.z, v.w};
  split_store(a, o, part, six);
}

// h = act(y + bias) written over y; with hs, also the split of h.  Same thread map as k_split3
// (the pad groups exist only when hs is written).
__global__ void __launch_bounds__(THREADS) k_bias_act_split(float* __restrict__ y, int64_t rows, int cols, int64_t ldy,
                                                            const float* __restrict__ bias, int act,
                                                            __nv_bfloat16* __restrict__ hs, int64_t ldhs, bool six) {
  const int part = hs ? part_of(cols) : cols;
  const int g = part >> 2;
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * g) return;
  const int64_t r = i / g;
  const int c = (int)(i % g) * 4;
  if (c >= cols) {
    zero_store(hs + r * ldhs + c, part, six);
    return;
  }
  float4* yp = reinterpret_cast<float4*>(y + r * ldy + c);
  const float4 v = *yp;
  const float4 b = *reinterpret_cast<const float4*>(bias + c);
  const float a[4] = {act_fwd(__fadd_rn(v.x, b.x), act), act_fwd(__fadd_rn(v.y, b.y), act),
                      act_fwd(__fadd_rn(v.z, b.z), act), act_fwd(__fadd_rn(v.w, b.w), act)};
  *yp = make_float4(a[0], a[1], a[2], a[3]);
  if (hs) split_store(a, hs + r * ldhs + c, part, six);
}

// h = act(y + bias) written over y and the value head on it, v[r] = sum_c h[r][c] wv[c] + bv[0]
// (a hidden layer followed by a width-1 Linear): one warp per row, 16-byte column groups.
__global__ void __launch_bounds__(THREADS) k_bias_act_value(float* __restrict__ y, int64_t rows, int cols, int64_t ldy,
                                                            const float* __restrict__ bias, int act,
                                                            const float* __restrict__ wv, const float* __restrict__ bv,
                                                            float* __restrict__ v) {
  const int lane = threadIdx.x & 31;
  const int64_t r = ((int64_t)blockIdx.x * THREADS + threadIdx.x) >> 5;
  if (r >= rows) return;
  float acc = 0.0f;
  for (int c = lane * 4; c < cols; c += 128) {
    float4* yp = reinterpret_cast<float4*>(y + r * ldy + c);
    const float4 t = *yp;
    const float4 b = *reinterpret_cast<const float4*>(bias + c);
    const float4 w = *reinterpret_cast<const float4*>(wv + c);
    const float4 h = make_float4(act_fwd(__fadd_rn(t.x, b.x), act), act_fwd(__fadd_rn(t.y, b.y), act),
                                 act_fwd(__fadd_rn(t.z, b.z), act), act_fwd(__fadd_rn(t.w, b.w), act));
    *yp = h;
    acc = __fmaf_rn(h.x, w.x, acc);
    acc = __fmaf_rn(h.y, w.y, acc);
    acc = __fmaf_rn(h.z, w.z, acc);
    acc = __fmaf_rn(h.w, w.w, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
  if (lane == 0) v[r] = __fadd_rn(acc, bv[0]);
}

// g_y = act'(g_h, h), its split, and the column sums of g_y over the block's rows.  A block is
// RS row slots x G column groups of 4 (G = part / 4 <= THREADS, RS = THREADS / G); block b owns
// rows [b rpb, (b + 1) rpb), slot s walks rows s, s + RS, ...; each thread sums its column group
// in row order and the slots are added in slot order, so the partial sums are deterministic.
__global__ void __launch_bounds__(THREADS) k_act_grad_split(const float* __restrict__ gh, int64_t ldg,
                                                            const float* __restrict__ h, int64_t ldh, int64_t rows,
                                                            int cols, int act, __nv_bfloat16* __restrict__ gys,
                                                            int64_t ldgs, float* __restrict__ col_part, int64_t rpb,
                                                            const float* __restrict__ gv, const float* __restrict__ wv,
                                                            float* __restrict__ v_part, bool six) {
  __shared__ float4 red[THREADS];
  __shared__ float4 red_v[THREADS];
  const int part = part_of(cols);
  const int G = part >> 2;
  const int RS = THREADS / G;
  const int tid = threadIdx.x;
  const int slot = tid / G;
  const int c = (tid % G) * 4;
  float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float4 acc_v = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  const float4 w = (gv && c < cols) ? *reinterpret_cast<const float4*>(wv + c) : acc;
  if (slot < RS) {
    const int64_t r0 = (int64_t)blockIdx.x * rpb;
    const int64_t r1 = r0 + rpb < rows ? r0 + rpb : rows;
    // GRAD_UNROLL rows per pass: all their loads are issued before any is used, so each thread
    // keeps several 16-byte loads in flight; rows are still summed in order r, r + RS, ...
    for (int64_t rb = r0 + slot; rb < r1; rb += (int64_t)GRAD_UNROLL * RS) {
      float4 gl[GRAD_UNROLL], hl[GRAD_UNROLL];
      float gr[GRAD_UNROLL];
#pragma unroll
      for (int u = 0; u < GRAD_UNROLL; u++) {
        const int64_t r = rb + (int64_t)u * RS;
        gr[u] = 0.0f;
        gl[u] = hl[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (r >= r1 || c >= cols) continue;
        if (gv) {   // the value head's input gradient g_v[r] wv[c], formed here instead of read
          gr[u] = gv[r];
          gl[u] = make_float4(__fmul_rn(gr[u], w.x), __fmul_rn(gr[u], w.y), __fmul_rn(gr[u], w.z),
                              __fmul_rn(gr[u], w.w));
        } else {
          gl[u] = *reinterpret_cast<const float4*>(gh + r * ldg + c);
        }
        hl[u] = act == F16_ACT_NONE && !gv ? gl[u] : *reinterpret_cast<const float4*>(h + r * ldh + c);
      }
#pragma unroll
      for (int u = 0; u < GRAD_UNROLL; u++) {
        const int64_t r = rb + (int64_t)u * RS;
        if (r >= r1) break;
        __nv_bfloat16* o = gys + r * ldgs + c;
        if (c >= cols) {
          zero_store(o, part, six);
          continue;
        }
        const float4 g = gl[u], hv = hl[u];
        const float a[4] = {act_bwd(g.x, hv.x, act), act_bwd(g.y, hv.y, act), act_bwd(g.z, hv.z, act),
                            act_bwd(g.w, hv.w, act)};
        acc.x = __fadd_rn(acc.x, a[0]);
        acc.y = __fadd_rn(acc.y, a[1]);
        acc.z = __fadd_rn(acc.z, a[2]);
        acc.w = __fadd_rn(acc.w, a[3]);
        if (gv) {   // the value weight's gradient: column sums of g_v[r] h[r][c]
          acc_v.x = __fmaf_rn(gr[u], hv.x, acc_v.x);
          acc_v.y = __fmaf_rn(gr[u], hv.y, acc_v.y);
          acc_v.z = __fmaf_rn(gr[u], hv.z, acc_v.z);
          acc_v.w = __fmaf_rn(gr[u], hv.w, acc_v.w);
        }
        split_store(a, o, part, six);
      }
    }
  }
  red[tid] = acc;
  red_v[tid] = acc_v;
  __syncthreads();
  if (tid < G && c < cols) {
    float4 s = red[tid], sv = red_v[tid];
    for (int j = 1; j < RS; j++) {
      const float4 t = red[j * G + tid], tv = red_v[j * G + tid];
      s.x = __fadd_rn(s.x, t.x);
      s.y = __fadd_rn(s.y, t.y);
      s.z = __fadd_rn(s.z, t.z);
      s.w = __fadd_rn(s.w, t.w);
      sv.x = __fadd_rn(sv.x, tv.x);
      sv.y = __fadd_rn(sv.y, tv.y);
      sv.z = __fadd_rn(sv.z, tv.z);
      sv.w = __fadd_rn(sv.w, tv.w);
    }
    *reinterpret_cast<float4*>(col_part + (int64_t)blockIdx.x * cols + c) = s;
    if (gv) *reinterpret_cast<float4*>(v_part + (int64_t)blockIdx.x * cols + c) = sv;
  }
}

// ---- categorical head ----------------------------------------------------------------------
// torch.distributions.Categorical(logits=z.view(-1, A, B)) as the update evaluates it
// (R/claude_code/model.py:198-215): per group of B logits, l = z - logsumexp(z) (amax, an
// infinite max replaced by 0, log of the sum of exp(z - max), plus the max), p = softmax(l)
// (exp(l - max l) / sum), log_prob = l[action], entropy = -sum(max(l, -FLT_MAX) p); the row's
// log-prob and entropy are the sums over its A groups (in group order).  A block of CAT_THREADS
// threads takes R = CAT_THREADS / A rows, one thread per (row, group); the rows are staged in
// shared memory (16-byte loads when the layout allows) with an odd row stride.
constexpr int CAT_THREADS = 256;
constexpr int CAT_MAXB = 32;
constexpr int CAT_MAXW = 128;
constexpr int CAT_SMEM = CAT_THREADS * (CAT_MAXB + 1);   // >= R (W + 1) for every A, B allowed

__device__ __forceinline__ void cat_stage(float* s, const float* __restrict__ z, int64_t ldz, int nrow, int W,
                                          int64_t r0, bool vec) {
  if (vec) {
    const int w4 = W >> 2;
    for (int i = threadIdx.x; i < nrow * w4; i += blockDim.x) {
      const int r = i / w4, c = (i - r * w4) * 4;
      const float4 v = *reinterpret_cast<const float4*>(z + (r0 + r) * ldz + c);
      float* d = s + r * (W + 1) + c;
      d[0] = v.x;
      d[1] = v.y;
      d[2] = v.z;
      d[3] = v.w;
    }
  } else {
    for (int i = threadIdx.x; i < nrow * W; i += blockDim.x) {
      const int r = i / W, c = i - r * W;
      s[r * (W + 1) + c] = z[(r0 + r) * ldz + c];
    }
  }
}

__device__ __forceinline__ int64_t cat_action(const void* action, int act_bytes, int64_t i) {
  return act_bytes == 1 ? (int64_t) reinterpret_cast<const uint8_t*>(action)[i]
                        : reinterpret_cast<const int64_t*>(action)[i];
}

// l (normalised logits), p and the entropy H of one group of B <= NB logits held in l on entry.
template <int NB>
__device__ __forceinline__ float cat_group(float (&l)[NB], float (&p)[NB], int B, bool& nan) {
  float mx = -INFINITY;
#pragma unroll
  for (int j = 0; j < NB; j++)
    if (j < B) {
      nan |= l[j] != l[j];
      mx = fmaxf(mx, l[j]);
    }
  if (fabsf(mx) == INFINITY) mx = 0.0f;
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < NB; j++)
    if (j < B) sum = __fadd_rn(sum, expf(__fsub_rn(l[j], mx)));
  const float lse = __fadd_rn(logf(sum), mx);
  float m2 = -INFINITY;
#pragma unroll
  for (int j = 0; j < NB; j++)
    if (j < B) {
      l[j] = __fsub_rn(l[j], lse);
      m2 = fmaxf(m2, l[j]);
    }
  float s2 = 0.0f;
#pragma unroll
  for (int j = 0; j < NB; j++)
    if (j < B) {
      p[j] = expf(__fsub_rn(l[j], m2));
      s2 = __fadd_rn(s2, p[j]);
    }
  float acc = 0.0f;
#pragma unroll
  for (int j = 0; j < NB; j++)
    if (j < B) {
      p[j] = __fdiv_rn(p[j], s2);
      acc = __fadd_rn(acc, __fmul_rn(fmaxf(l[j], -FLT_MAX), p[j]));
    }
  return -acc;
}

template <int NB>
__global__ void __launch_bounds__(CAT_THREADS) k_cat_fwd(const float* __restrict__ z, int64_t ldz, int64_t M, int A,
                                                         int B, bool vec, const void* __restrict__ action,
                                                         int act_bytes, float* __restrict__ logp,
                                                         float* __restrict__ ent, int* __restrict__ flags) {
  __shared__ float s[CAT_SMEM];
  __shared__ float2 grp[CAT_THREADS];
  const int W = A * B, R = CAT_THREADS / A;
  const int64_t r0 = (int64_t)blockIdx.x * R;
  const int nrow = (int)(M - r0 < R ? M - r0 : R);
  cat_stage(s, z, ldz, nrow, W, r0, vec);
  __syncthreads();
  const int r = threadIdx.x / A, a = threadIdx.x - r * A;
  if (r < nrow) {
    float l[NB], p[NB];
    const float* row = s + r * (W + 1) + a * B;
#pragma unroll
    for (int j = 0; j < NB; j++) l[j] = j < B ? row[j] : 0.0f;
    bool nan = false;
    const float H = cat_group(l, p, B, nan);
    const int64_t act = cat_action(action, act_bytes, (r0 + r) * A + a);
    float lp = 0.0f;
#pragma unroll
    for (int j = 0; j < NB; j++)
      if (j == act) lp = l[j];
    grp[threadIdx.x] = make_float2(lp, H);
    const bool bad = act < 0 || act >= B;
    if (nan || bad) atomicOr(flags, (nan ? 1 : 0) | (bad ? 2 : 0));
  }
  __syncthreads();
  if (threadIdx.x < nrow) {
    float lp_sum = 0.0f, h_sum = 0.0f;
    for (int g = 0; g < A; g++) {
      const float2 v = grp[threadIdx.x * A + g];
      lp_sum = __fadd_rn(lp_sum, v.x);
      h_sum = __fadd_rn(h_sum, v.y);
    }
    logp[r0 + threadIdx.x] = lp_sum;
    ent[r0 + threadIdx.x] = h_sum;
  }
}

// dz = g_lp (onehot(action) - p) - g_ent p (max(l, -FLT_MAX) + H) per group (the gradient of
// g_lp log_prob + g_ent entropy through logsumexp, softmax and the clamp); absent upstream
// gradients count as zero.
template <int NB>
__global__ void __launch_bounds__(CAT_THREADS) k_cat_bwd(const float* __restrict__ z, int64_t ldz, int64_t M, int A,
                                                         int B, bool vec, const void* __restrict__ action,
                                                         int act_bytes, const float* __restrict__ g_lp,
                                                         const float* __restrict__ g_ent, float* __restrict__ gz,
                                                         int64_t ldg) {
  __shared__ float s[CAT_SMEM];
  const int W = A * B, R = CAT_THREADS / A;
  const int64_t r0 = (int64_t)blockIdx.x * R;
  const int nrow = (int)(M - r0 < R ? M - r0 : R);
  cat_stage(s, z, ldz, nrow, W, r0, vec);
  __syncthreads();
  const int r = threadIdx.x / A, a = threadIdx.x - r * A;
  if (r < nrow) {
    float* row = s + r * (W + 1) + a * B;
    const int64_t m = r0 + r;
    const float gl = g_lp ? g_lp[m] : 0.0f;
    const float ge = g_ent ? g_ent[m] : 0.0f;
    float l[NB], p[NB];
#pragma unroll
    for (int j = 0; j < NB; j++) l[j] = j < B ? row[j] : 0.0f;
    bool nan = false;
    const float H = cat_group(l, p, B, nan);
    const int64_t act = cat_action(action, act_bytes, m * A + a);
#pragma unroll
    for (int j = 0; j < NB; j++)
      if (j < B) {
        const float d = __fsub_rn(j == act ? 1.0f : 0.0f, p[j]);
        const float e = __fmul_rn(p[j], __fadd_rn(fmaxf(l[j], -FLT_MAX), H));
        row[j] = __fsub_rn(__fmul_rn(gl, d), __fmul_rn(ge, e));
      }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nrow * W; i += blockDim.x) {
    const int rr = i / W, c = i - rr * W;
    gz[(r0 + rr) * ldg + c] = s[rr * (W + 1) + c];
  }
}

inline unsigned grid_for(int64_t n) { return (unsigned)((n + THREADS - 1) / THREADS); }

}  // namespace upd
}  // namespace f16

using namespace f16;

extern "C" int f16_split3_bf16(const float* x, int64_t rows, int cols, int64_t ldx, void* out, int64_t ldo,
                               int parts, f16_stream_t stream) {
  if (!x || !out || rows <= 0 || cols <= 0 || cols % 4 || ldx < cols || (parts != 3 && parts != 6) ||
      ldo < parts * (int64_t)upd::part_of(cols))
    return F16_ERR_ARG;
  if (!aligned(x, 16) || ldx % 4 || !aligned(out, 8) || ldo % 4) return F16_ERR_ALIGN;
  const int64_t n = rows * (upd::part_of(cols) / 4);
  upd::k_split3<<<upd::grid_for(n), upd::THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, rows, cols, ldx, reinterpret_cast<__nv_bfloat16*>(out), ldo, parts == 6);
  return launch_status();
}

extern "C" int f16_bias_act_split(float* y, int64_t rows, int cols, int64_t ldy, const float* bias, int act,
                                  void* hs, int64_t ldhs, int parts, f16_stream_t stream) {
  if (!y || !bias || rows <= 0 || cols <= 0 || cols % 4 || ldy < cols || act < F16_ACT_NONE || act > F16_ACT_TANH)
    return F16_ERR_ARG;
  if (hs && ((parts != 3 && parts != 6) || ldhs < parts * (int64_t)upd::part_of(cols))) return F16_ERR_ARG;
  if (!aligned(y, 16) || ldy % 4 || !aligned(bias, 16) || (hs && (!aligned(hs, 8) || ldhs % 4))) return F16_ERR_ALIGN;
  const int64_t n = rows * ((hs ? upd::part_of(cols) : cols) / 4);
  upd::k_bias_act_split<<<upd::grid_for(n), upd::THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      y, rows, cols, ldy, bias, act, reinterpret_cast<__nv_bfloat16*>(hs), ldhs, parts == 6);
  return launch_status();
}

extern "C" int f16_act_grad_split(const float* gh, int64_t ldg, const float* h, int64_t ldh, int64_t rows, int cols,
                                  int act, void* gys, int64_t ldgs, int parts, float* col_part, int nblk,
                                  f16_stream_t stream) {
  if (!gh || !gys || !col_part || rows <= 0 || cols <= 0 || cols % 4 || cols > upd::MAX_GRAD_COLS || ldg < cols ||
      (parts != 3 && parts != 6) || ldgs < parts * (int64_t)upd::part_of(cols) || nblk <= 0 || act < F16_ACT_NONE ||
      act > F16_ACT_TANH)
    return F16_ERR_ARG;
  if (act != F16_ACT_NONE && (!h || ldh < cols)) return F16_ERR_ARG;
  if (!aligned(gh, 16) || ldg % 4 || !aligned(gys, 8) || ldgs % 4 || !aligned(col_part, 16) ||
      (act != F16_ACT_NONE && (!aligned(h, 16) || ldh % 4)))
    return F16_ERR_ALIGN;
  const int64_t rpb = (rows + nblk - 1) / nblk;
  upd::k_act_grad_split<<<(unsigned)nblk, upd::THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      gh, ldg, h, ldh, rows, cols, act, reinterpret_cast<__nv_bfloat16*>(gys), ldgs, col_part, rpb, nullptr, nullptr,
      nullptr, parts == 6);
  return launch_status();
}

extern "C" int f16_bias_act_value(float* y, int64_t rows, int cols, int64_t ldy, const float* bias, int act,
                                  const float* wv, const float* bv, float* v, f16_stream_t stream) {
  if (!y || !bias || !wv || !bv || !v || rows <= 0 || cols <= 0 || cols % 4 || ldy < cols || act < F16_ACT_NONE ||
      act > F16_ACT_TANH)
    return F16_ERR_ARG;
  if (!aligned(y, 16) || ldy % 4 || !aligned(bias, 16) || !aligned(wv, 16)) return F16_ERR_ALIGN;
  const int64_t threads = rows * 32;
  upd::k_bias_act_value<<<upd::grid_for(threads), upd::THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      y, rows, cols, ldy, bias, act, wv, bv, v);
  return launch_status();
}

extern "C" int f16_act_grad_split_value(const float* gv, const float* wv, const float* h, int64_t ldh, int64_t rows,
                                        int cols, int act, void* gys, int64_t ldgs, int parts, float* col_part,
                                        float* v_part, int nblk, f16_stream_t stream) {
  if (!gv || !wv || !h || !gys || !col_part || !v_part || rows <= 0 || cols <= 0 || cols % 4 ||
      cols > upd::MAX_GRAD_COLS || ldh < cols || (parts != 3 && parts != 6) ||
      ldgs < parts * (int64_t)upd::part_of(cols) || nblk <= 0 || act < F16_ACT_NONE || act > F16_ACT_TANH)
    return F16_ERR_ARG;
  if (!aligned(wv, 16) || !aligned(h, 16) || ldh % 4 || !aligned(gys, 8) || ldgs % 4 || !aligned(col_part, 16) ||
      !aligned(v_part, 16))
    return F16_ERR_ALIGN;
  const int64_t rpb = (rows + nblk - 1) / nblk;
  upd::k_act_grad_split<<<(unsigned)nblk, upd::THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      nullptr, 0, h, ldh, rows, cols, act, reinterpret_cast<__nv_bfloat16*>(gys), ldgs, col_part, rpb, gv, wv, v_part,
      parts == 6);
  return launch_status();
}

static int cat_check(const float* z, int64_t ldz, int64_t M, int A, int B, const void* action, int act_bytes) {
  if (!z || !action || M <= 0 || A <= 0 || B <= 0 || B > upd::CAT_MAXB || A * B > upd::CAT_MAXW ||
      A > upd::CAT_THREADS || ldz < A * B ||
      (act_bytes != 1 && act_bytes != 8))
    return F16_ERR_ARG;
  if (!aligned(z, 4) || (act_bytes == 8 && !aligned(action, 8))) return F16_ERR_ALIGN;
  return F16_OK;
}

static bool cat_vec(const float* z, int64_t ldz, int W) { return W % 4 == 0 && ldz % 4 == 0 && aligned(z, 16); }

extern "C" int f16_categorical_fwd(const float* logits, int64_t ldz, int64_t M, int A, int B, const void* action,
                                   int act_bytes, float* logp, float* ent, int* flags, f16_stream_t stream) {
  const int rc = cat_check(logits, ldz, M, A, B, action, act_bytes);
  if (rc != F16_OK) return rc;
  if (!logp || !ent || !flags) return F16_ERR_ARG;
  const int R = upd::CAT_THREADS / A;
  const unsigned grid = (unsigned)((M + R - 1) / R);
  auto k = B == 21 ? upd::k_cat_fwd<21> : upd::k_cat_fwd<upd::CAT_MAXB>;   // the reference's 21 bins, exact size
  k<<<grid, upd::CAT_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, ldz, M, A, B, cat_vec(logits, ldz, A * B), action, act_bytes, logp, ent, flags);
  return launch_status();
}

extern "C" int f16_categorical_bwd(const float* logits, int64_t ldz, int64_t M, int A, int B, const void* action,
                                   int act_bytes, const float* g_lp, const float* g_ent, float* gz, int64_t ldg,
                                   f16_stream_t stream) {
  const int rc = cat_check(logits, ldz, M, A, B, action, act_bytes);
  if (rc != F16_OK) return rc;
  if (!gz || ldg < A * B) return F16_ERR_ARG;
  const int R = upd::CAT_THREADS / A;
  const unsigned grid = (unsigned)((M + R - 1) / R);
  auto k = B == 21 ? upd::k_cat_bwd<21> : upd::k_cat_bwd<upd::CAT_MAXB>;
  k<<<grid, upd::CAT_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      logits, ldz, M, A, B, cat_vec(logits, ldz, A * B), action, act_bytes, g_lp, g_ent, gz, ldg);
  return launch_status();
}
