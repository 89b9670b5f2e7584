// rollout_kernels.cu -- GAE and observation running-normalisation kernels with their C ABI.
//
// GAE (R/cuda_fdm/ppo_gpu.py:1983-1995): the reference runs T rounds of fp32 torch elementwise
// ops.  Here one thread owns one environment column and walks t = T-1..0 in registers; each
// operation is rounded exactly as the corresponding torch op (explicit __f*_rn, no contraction,
// Python scalars cast to float as torch's float opmath does), so the result is bit-identical to
// the reference while the whole rollout buffer is read once (20 bytes per (t, env)).
//
// RunningNorm (ppo_gpu.py:184-222): batch mean / population variance per feature reduced in fp64
// (two kernels: per-block partial sums, then a per-feature combine that applies the reference's
// Chan merge in fp32), and the normalise-clamp that produces the policy input, optionally also
// as a zero-padded bf16 matrix (the MLP kernel's A operand).
#include <cuda_bf16.h>
#include <mutex>
#include "common.cuh"

namespace f16 {
namespace ro {

constexpr int GAE_THREADS = 256;

__global__ void __launch_bounds__(GAE_THREADS)
k_gae(const float* __restrict__ rew, const float* __restrict__ val, const float* __restrict__ done,
      const float* __restrict__ last_val, const float* __restrict__ next_done, int T, int64_t n, int64_t ld,
      float g, float gl, float* __restrict__ adv, float* __restrict__ ret) {
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  float lastgae = 0.0f;
  float nv = last_val[e];
  float nnt = __fsub_rn(1.0f, next_done[e]);
  for (int t = T - 1; t >= 0; t--) {
    int64_t i = (int64_t)t * ld + e;
    float r = rew[i], v = val[i];
    // delta = rew[t] + gamma * next_values * next_nonterminal - val[t]
    float delta = __fsub_rn(__fadd_rn(r, __fmul_rn(__fmul_rn(g, nv), nnt)), v);
    // lastgae = delta + gamma * lambda * next_nonterminal * lastgae
    lastgae = __fadd_rn(delta, __fmul_rn(__fmul_rn(gl, nnt), lastgae));
    adv[i] = lastgae;
    ret[i] = __fadd_rn(lastgae, v);
    nv = v;
    nnt = __fsub_rn(1.0f, done[i]);
  }
}

constexpr int NORM_THREADS = 256;
constexpr int NORM_ROWS_PER_BLOCK = 512;

// partial[b][d] = (sum, sum of squares) over this block's rows, fp64
__global__ void __launch_bounds__(NORM_THREADS)
k_norm_partial(const float* __restrict__ x, int64_t B, int D, int64_t ldx, double2* __restrict__ partial) {
  int64_t r0 = (int64_t)blockIdx.x * NORM_ROWS_PER_BLOCK;
  int64_t r1 = r0 + NORM_ROWS_PER_BLOCK < B ? r0 + NORM_ROWS_PER_BLOCK : B;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    double s = 0.0, q = 0.0;
    for (int64_t r = r0; r < r1; r++) {
      double v = (double)x[r * ldx + d];
      s += v;
      q += v * v;
    }
    partial[(int64_t)blockIdx.x * D + d] = make_double2(s, q);
  }
}

// combine the partials and apply the reference's Chan merge (all fp32 ops, reference order):
//   delta = b_mean - mean; tot = count + b_count; mean += delta * (b_count / tot)
//   M2 = var*count + b_var*b_count + (delta*delta) * (count*b_count / tot); var = M2 / tot
__global__ void __launch_bounds__(NORM_THREADS)
k_norm_merge(const double2* __restrict__ partial, int nblk, int64_t B, int D, float* __restrict__ mean,
             float* __restrict__ var, float* __restrict__ count) {
  int d = blockIdx.x * blockDim.x + threadIdx.x;
  float c = count[0];
  float bc = (float)B;
  float tot = __fadd_rn(c, bc);
  __syncthreads();
  if (d < D) {
    double s = 0.0, q = 0.0;
    for (int b = 0; b < nblk; b++) {
      double2 p = partial[(int64_t)b * D + d];
      s += p.x;
      q += p.y;
    }
    double m = s / (double)B;
    double vv = q / (double)B - m * m;
    float bm = (float)m, bv = (float)(vv > 0.0 ? vv : 0.0);
    float mu = mean[d], va = var[d];
    float delta = __fsub_rn(bm, mu);
    mean[d] = __fadd_rn(mu, __fmul_rn(delta, __fdiv_rn(bc, tot)));
    float M2 = __fadd_rn(__fadd_rn(__fmul_rn(va, c), __fmul_rn(bv, bc)),
                         __fmul_rn(__fmul_rn(delta, delta), __fdiv_rn(__fmul_rn(c, bc), tot)));
    var[d] = __fdiv_rn(M2, tot);
  }
}

// sums[d] = sum over the partial rows (same order as k_norm_merge, so a merge of sums reproduces
// f16_norm_update bit for bit on one device)
__global__ void __launch_bounds__(NORM_THREADS)
k_norm_reduce(const double2* __restrict__ partial, int nblk, int D, double2* __restrict__ sums) {
  int d = blockIdx.x * blockDim.x + threadIdx.x;
  if (d >= D) return;
  double s = 0.0, q = 0.0;
  for (int b = 0; b < nblk; b++) {
    double2 p = partial[(int64_t)b * D + d];
    s += p.x;
    q += p.y;
  }
  sums[d] = make_double2(s, q);
}

__global__ void k_norm_count(float* __restrict__ count, int64_t B) {
  if (threadIdx.x == 0 && blockIdx.x == 0) count[0] = __fadd_rn(count[0], (float)B);
}

// y = clamp((x - mean) / sqrt(var + eps), -clip, clip); fp32 out and/or bf16 out padded to ldb
// columns (zeros beyond D).
__global__ void __launch_bounds__(NORM_THREADS)
k_norm_apply(const float* __restrict__ x, int64_t B, int D, int64_t ldx, const float* __restrict__ mean,
             const float* __restrict__ var, float eps, float clip, float* __restrict__ y, int64_t ldy,
             __nv_bfloat16* __restrict__ yb, int64_t ldb) {
  int64_t r = blockIdx.y;
  for (int64_t rr = r; rr < B; rr += gridDim.y) {
    for (int d = blockIdx.x * blockDim.x + threadIdx.x; d < (yb ? ldb : D); d += gridDim.x * blockDim.x) {
      float o = 0.0f;
      if (d < D) {
        float den = __fsqrt_rn(__fadd_rn(var[d], eps));
        o = __fdiv_rn(__fsub_rn(x[rr * ldx + d], mean[d]), den);
        o = o < -clip ? -clip : (o > clip ? clip : o);     // torch.clamp_: NaN stays NaN
        if (y) y[rr * ldy + d] = o;
      }
      if (yb) yb[rr * ldb + d] = __float2bfloat16_rn(o);
    }
  }
}

}  // namespace ro
}  // namespace f16

using namespace f16;

extern "C" int f16_gae(const float* rew, const float* val, const float* done, const float* last_val,
                       const float* next_done, int T, int64_t n, int64_t ld, double gamma, double lam, float* adv,
                       float* ret, f16_stream_t stream) {
  if (!rew || !val || !done || !last_val || !next_done || !adv || !ret || T <= 0 || n <= 0 || ld < n)
    return F16_ERR_ARG;
  float g = (float)gamma;
  float gl = (float)(gamma * lam);       // Python evaluates gamma * gae_lambda in double first
  int grid = (int)((n + ro::GAE_THREADS - 1) / ro::GAE_THREADS);
  ro::k_gae<<<grid, ro::GAE_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(rew, val, done, last_val,
                                                                                   next_done, T, n, ld, g, gl, adv,
                                                                                   ret);
  return launch_status();
}

extern "C" int f16_norm_update(const float* x, int64_t B, int D, int64_t ldx, float* mean, float* var, float* count,
                               double* scratch, int64_t scratch_doubles, f16_stream_t stream) {
  if (!x || !mean || !var || !count || !scratch || B <= 0 || D <= 0 || ldx < D) return F16_ERR_ARG;
  int nblk = (int)((B + ro::NORM_ROWS_PER_BLOCK - 1) / ro::NORM_ROWS_PER_BLOCK);
  if (scratch_doubles < (int64_t)nblk * D * 2) return F16_ERR_TOO_LARGE;
  if (!aligned(scratch, 16)) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  double2* part = reinterpret_cast<double2*>(scratch);
  ro::k_norm_partial<<<nblk, ro::NORM_THREADS, 0, s>>>(x, B, D, ldx, part);
  ro::k_norm_merge<<<(D + ro::NORM_THREADS - 1) / ro::NORM_THREADS, ro::NORM_THREADS, 0, s>>>(part, nblk, B, D,
                                                                                            mean, var, count);
  ro::k_norm_count<<<1, 32, 0, s>>>(count, B);
  return launch_status();
}

extern "C" int f16_norm_sums(const float* x, int64_t B, int D, int64_t ldx, double* sums, double* scratch,
                             int64_t scratch_doubles, f16_stream_t stream) {
  if (!x || !sums || !scratch || B <= 0 || D <= 0 || ldx < D) return F16_ERR_ARG;
  int nblk = (int)((B + ro::NORM_ROWS_PER_BLOCK - 1) / ro::NORM_ROWS_PER_BLOCK);
  if (scratch_doubles < (int64_t)nblk * D * 2) return F16_ERR_TOO_LARGE;
  if (!aligned(scratch, 16) || !aligned(sums, 16)) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  double2* part = reinterpret_cast<double2*>(scratch);
  ro::k_norm_partial<<<nblk, ro::NORM_THREADS, 0, s>>>(x, B, D, ldx, part);
  ro::k_norm_reduce<<<(D + ro::NORM_THREADS - 1) / ro::NORM_THREADS, ro::NORM_THREADS, 0, s>>>(
      part, nblk, D, reinterpret_cast<double2*>(sums));
  return launch_status();
}

extern "C" int f16_norm_merge_sums(const double* sums, int64_t B_total, int D, float* mean, float* var,
                                   float* count, f16_stream_t stream) {
  if (!sums || !mean || !var || !count || B_total <= 0 || D <= 0) return F16_ERR_ARG;
  if (!aligned(sums, 16)) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  ro::k_norm_merge<<<(D + ro::NORM_THREADS - 1) / ro::NORM_THREADS, ro::NORM_THREADS, 0, s>>>(
      reinterpret_cast<const double2*>(sums), 1, B_total, D, mean, var, count);
  ro::k_norm_count<<<1, 32, 0, s>>>(count, B_total);
  return launch_status();
}

extern "C" int64_t f16_norm_scratch_doubles(int64_t B, int D) {
  int64_t nblk = (B + ro::NORM_ROWS_PER_BLOCK - 1) / ro::NORM_ROWS_PER_BLOCK;
  return nblk * D * 2;
}

extern "C" int f16_norm_apply(const float* x, int64_t B, int D, int64_t ldx, const float* mean, const float* var,
                              double eps, double clip, float* y, int64_t ldy, void* y_bf16, int64_t ldb,
                              f16_stream_t stream) {
  if (!x || !mean || !var || B <= 0 || D <= 0 || ldx < D || (!y && !y_bf16)) return F16_ERR_ARG;
  if ((y && ldy < D) || (y_bf16 && ldb < D)) return F16_ERR_ARG;
  dim3 grid((unsigned)(((y_bf16 ? ldb : D) + ro::NORM_THREADS - 1) / ro::NORM_THREADS),
            (unsigned)(B < 65535 ? B : 65535));
  ro::k_norm_apply<<<grid, ro::NORM_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      x, B, D, ldx, mean, var, (float)eps, (float)clip, y, ldy, reinterpret_cast<__nv_bfloat16*>(y_bf16), ldb);
  return launch_status();
}

// ---------------------------------------------------------------------------------------------
// RunningNorm update with library-owned scratch (no counterpart in the reference).
//
// For callers that cannot allocate device memory at the point of the update: a fixed-size
// memory pool or arena that is sealed once training starts, or a host driver that forbids
// allocation inside its step loop.  The fp64 partial sums live in a file-scope device array of
// F16_NORM_STATIC_SCRATCH_PAIRS double2 (2 MiB) instead of a caller buffer; its address is read
// once per device with cudaGetSymbolAddress.  Every scratch slot that the merge kernel reads is
// written by the partial kernel of the same call first, so nothing needs to start at zero.
// There is one array per device, so two calls in flight at the same time on one device (two
// streams, or two host threads) race on it; calls queued on one stream are ordered and safe.
// ---------------------------------------------------------------------------------------------
static __device__ __align__(256) double2 g_norm_static_scratch[F16_NORM_STATIC_SCRATCH_PAIRS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_norm_static_mu;
double2* g_norm_static_addr[kMaxDevices] = {};

// Device address of g_norm_static_scratch on the current device (looked up on first use).
int norm_static_scratch(double2** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return F16_ERR_CUDA;
  std::lock_guard<std::mutex> lock(g_norm_static_mu);
  if (!g_norm_static_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_norm_static_scratch) != cudaSuccess || !p) {
      cudaGetLastError();
      return F16_ERR_CUDA;
    }
    g_norm_static_addr[dev] = static_cast<double2*>(p);
  }
  *out = g_norm_static_addr[dev];
  return F16_OK;
}
}  // namespace

extern "C" int f16_norm_update_static(const float* x, int64_t B, int D, int64_t ldx, float* mean, float* var,
                                      float* count, f16_stream_t stream) {
  if (!x || !mean || !var || !count || B <= 0 || D <= 0 || ldx < D) return F16_ERR_ARG;
  int64_t nblk = (B + ro::NORM_ROWS_PER_BLOCK - 1) / ro::NORM_ROWS_PER_BLOCK;
  if (nblk * D > (int64_t)F16_NORM_STATIC_SCRATCH_PAIRS) return F16_ERR_TOO_LARGE;
  double2* part = nullptr;
  int rc = norm_static_scratch(&part);
  if (rc != F16_OK) return rc;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  ro::k_norm_partial<<<(unsigned)nblk, ro::NORM_THREADS, 0, s>>>(x, B, D, ldx, part);
  ro::k_norm_merge<<<(D + ro::NORM_THREADS - 1) / ro::NORM_THREADS, ro::NORM_THREADS, 0, s>>>(
      part, (int)nblk, B, D, mean, var, count);
  ro::k_norm_count<<<1, 32, 0, s>>>(count, B);
  return launch_status();
}
