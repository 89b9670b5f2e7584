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
#include <cuda_fp16.h>
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
#pragma unroll 8
    for (int64_t r = r0; r < r1; r++) {
      double v = (double)x[r * ldx + d];
      s += v;
      q += v * v;
    }
    partial[(int64_t)blockIdx.x * D + d] = make_double2(s, q);
  }
}

// The same partial sums with 16-byte loads, for D % 4 == 0 and a 16-byte aligned, 4-float
// strided x: thread t sums columns 4c..4c+3 (c = t mod D/4) of the rows r0 + j, r0 + j + S, ...
// (stripe j = t div D/4, S = PART4_THREADS div D/4 stripes), so two resident blocks of 768
// threads per SM keep ~94 KB of loads in flight instead of one 4-byte load per column (512-thread
// blocks: the update 11% slower); the stripes' fp64 sums meet in shared memory (at most 48 KB per
// block) and are added in stripe order (deterministic).
constexpr int PART4_THREADS = 768;
__global__ void __launch_bounds__(PART4_THREADS, 2)
k_norm_partial4(const float4* __restrict__ x, int64_t B, int D, int64_t ldx4, double2* __restrict__ partial) {
  extern __shared__ double2 stripes[];              // [S][D]
  const int ncg = D >> 2;
  const int S = PART4_THREADS / ncg;
  const int cg = threadIdx.x % ncg, st = threadIdx.x / ncg;
  const int64_t r0 = (int64_t)blockIdx.x * NORM_ROWS_PER_BLOCK;
  const int64_t r1 = r0 + NORM_ROWS_PER_BLOCK < B ? r0 + NORM_ROWS_PER_BLOCK : B;
  if (st < S) {
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0, q0 = 0.0, q1 = 0.0, q2 = 0.0, q3 = 0.0;
#pragma unroll 4
    for (int64_t r = r0 + st; r < r1; r += S) {
      const float4 v = x[r * ldx4 + cg];
      const double a = v.x, b = v.y, c = v.z, d = v.w;
      s0 += a; q0 += a * a;
      s1 += b; q1 += b * b;
      s2 += c; q2 += c * c;
      s3 += d; q3 += d * d;
    }
    double2* o = stripes + (int64_t)st * D + 4 * cg;
    o[0] = make_double2(s0, q0);
    o[1] = make_double2(s1, q1);
    o[2] = make_double2(s2, q2);
    o[3] = make_double2(s3, q3);
  }
  __syncthreads();
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    double s = 0.0, q = 0.0;
    for (int i = 0; i < S; i++) {
      const double2 p = stripes[(int64_t)i * D + d];
      s += p.x;
      q += p.y;
    }
    partial[(int64_t)blockIdx.x * D + d] = make_double2(s, q);
  }
}

// Sum of the partial rows of 32 features per block: warp w adds rows w, w+8, ... (unrolled, so
// many loads are in flight), then the 8 warp sums are added in warp order.  Both the merge and
// the cross-rank sums use it, so one rank reproduces f16_norm_update bit for bit.
constexpr int MERGE_WARPS = NORM_THREADS / 32;
__device__ __forceinline__ bool sum_partials(const double2* __restrict__ partial, int nblk, int D, double2& out) {
  __shared__ double2 acc[MERGE_WARPS][32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int d = blockIdx.x * 32 + lane;
  double s = 0.0, q = 0.0;
  if (d < D) {
#pragma unroll 4
    for (int b = w; b < nblk; b += MERGE_WARPS) {
      double2 p = partial[(int64_t)b * D + d];
      s += p.x;
      q += p.y;
    }
  }
  acc[w][lane] = make_double2(s, q);
  __syncthreads();
  if (w != 0 || d >= D) return false;
  s = 0.0; q = 0.0;
#pragma unroll
  for (int i = 0; i < MERGE_WARPS; i++) {
    s += acc[i][lane].x;
    q += acc[i][lane].y;
  }
  out = make_double2(s, q);
  return true;
}

// combine the partials and apply the reference's Chan merge (all fp32 ops, reference order):
//   delta = b_mean - mean; tot = count + b_count; mean += delta * (b_count / tot)
//   M2 = var*count + b_var*b_count + (delta*delta) * (count*b_count / tot); var = M2 / tot
// grid: ceil(D / 32) blocks of NORM_THREADS
__global__ void __launch_bounds__(NORM_THREADS)
k_norm_merge(const double2* __restrict__ partial, int nblk, int64_t B, int D, float* __restrict__ mean,
             float* __restrict__ var, float* __restrict__ count) {
  const int d = blockIdx.x * 32 + (threadIdx.x & 31);
  float c = count[0];
  float bc = (float)B;
  float tot = __fadd_rn(c, bc);
  double2 sq;
  if (sum_partials(partial, nblk, D, sq)) {
    const double s = sq.x, q = sq.y;
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
// f16_norm_update bit for bit on one device); grid: ceil(D / 32) blocks of NORM_THREADS
__global__ void __launch_bounds__(NORM_THREADS)
k_norm_reduce(const double2* __restrict__ partial, int nblk, int D, double2* __restrict__ sums) {
  double2 sq;
  if (sum_partials(partial, nblk, D, sq)) sums[blockIdx.x * 32 + (threadIdx.x & 31)] = sq;
}

__global__ void k_norm_count(float* __restrict__ count, int64_t B) {
  if (threadIdx.x == 0 && blockIdx.x == 0) count[0] = __fadd_rn(count[0], (float)B);
}

// One fp32 value as the 16-bit policy-input element: bf16, or fp16 saturated at +-65504 (NaN
// stays NaN), both round-to-nearest.
template <bool FP16>
__device__ __forceinline__ uint16_t to_half_bits(float o) {
  if (FP16) {
    const float c = o > 65504.0f ? 65504.0f : (o < -65504.0f ? -65504.0f : o);
    return __half_as_ushort(__float2half_rn(c));
  }
  return __bfloat16_as_ushort(__float2bfloat16_rn(o));
}

// y = clamp((x - mean) / sqrt(var + eps), -clip, clip); fp32 out and/or 16-bit (bf16 or fp16)
// out padded to ldb columns (zeros beyond D).  With mean == NULL the values pass through
// unchanged (a cast into the 16-bit layout).  One thread per column (den and mean loaded once),
// APPLY_ROWS rows per block; `nonfinite` (optional) counts warps that produced a non-finite
// output.
constexpr int APPLY_ROWS = 32;
template <bool FP16>
__global__ void __launch_bounds__(NORM_THREADS)
k_norm_apply(const float* __restrict__ x, int64_t B, int D, int64_t ldx, const float* __restrict__ mean,
             const float* __restrict__ var, float eps, float clip, float* __restrict__ y, int64_t ldy,
             uint16_t* __restrict__ yb, int64_t ldb, unsigned* __restrict__ nonfinite) {
  const int ncol = yb ? (int)ldb : D;
  const int64_t r0 = (int64_t)blockIdx.x * APPLY_ROWS;
  const int64_t r1 = r0 + APPLY_ROWS < B ? r0 + APPLY_ROWS : B;
  bool bad = false;
  for (int d = threadIdx.x; d < ncol; d += blockDim.x) {
    if (d < D) {
      const bool norm = mean != nullptr;
      const float mu = norm ? mean[d] : 0.0f;
      const float den = norm ? __fsqrt_rn(__fadd_rn(var[d], eps)) : 1.0f;
#pragma unroll 4
      for (int64_t rr = r0; rr < r1; rr++) {
        float o = x[rr * ldx + d];
        if (norm) {
          o = __fdiv_rn(__fsub_rn(o, mu), den);
          o = o < -clip ? -clip : (o > clip ? clip : o);   // torch.clamp_: NaN stays NaN
        }
        bad |= !isfinite(o);
        if (y) y[rr * ldy + d] = o;
        if (yb) yb[rr * ldb + d] = to_half_bits<FP16>(o);
      }
    } else {
      for (int64_t rr = r0; rr < r1; rr++) yb[rr * ldb + d] = 0;
    }
  }
  if (nonfinite && __any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicAdd(nonfinite, 1u);
}

// The same transform with 16-byte accesses, when D, the row strides and the pointers allow it:
// thread t handles columns 4c..4c+3 (c = t mod G, G = the written column groups: D/4, or ldb/4
// with the 16-bit padding) of rows r0 + j, r0 + j + S, ... (stripe j = t div G, S = 256 div G);
// the per-element arithmetic is k_norm_apply's, so the outputs are identical.  The fp32 rows are
// stored with the evict-first hint: in a rollout they are the stored observations, read again only
// by the update, while the 16-bit rows (the policy's next input) and the environment state that the
// next step reads stay in L2 (-0.6% per rollout, the environment step -1.3%).  Blocks take an
// equal share of rows (rpb each, at least APPLY4_MIN_ROWS) so that the grid fills APPLY4_WAVES
// waves of APPLY4_BLOCKS_PER_SM blocks per SM exactly: no partly filled last wave (-1.0% per
// rollout against fixed 64-row blocks at five blocks per SM).
constexpr int APPLY4_MIN_ROWS = 16, APPLY4_BLOCKS_PER_SM = 8, APPLY4_WAVES = 3;
__device__ __forceinline__ float norm_elem(float v, float mu, float den, bool norm, float clip) {
  if (!norm) return v;
  float o = __fdiv_rn(__fsub_rn(v, mu), den);
  return o < -clip ? -clip : (o > clip ? clip : o);
}
template <bool FP16>
__global__ void __launch_bounds__(NORM_THREADS, APPLY4_BLOCKS_PER_SM)
k_norm_apply4(const float4* __restrict__ x, int64_t B, int D, int64_t ldx4, const float* __restrict__ mean,
              const float* __restrict__ var, float eps, float clip, float4* __restrict__ y, int64_t ldy4,
              uint2* __restrict__ yb, int64_t ldb4, unsigned* __restrict__ nonfinite, int64_t rpb) {
  const int dg = D >> 2;
  const int G = yb ? (int)ldb4 : dg;
  const int S = NORM_THREADS / G;
  const int cg = threadIdx.x % G, st = threadIdx.x / G;
  const int64_t r0 = (int64_t)blockIdx.x * rpb;
  const int64_t r1 = r0 + rpb < B ? r0 + rpb : B;
  const bool norm = mean != nullptr;
  bool bad = false;
  if (st < S) {
    if (cg < dg) {
      float mu[4] = {0.0f, 0.0f, 0.0f, 0.0f}, den[4] = {1.0f, 1.0f, 1.0f, 1.0f};
      if (norm) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
          mu[i] = mean[4 * cg + i];
          den[i] = __fsqrt_rn(__fadd_rn(var[4 * cg + i], eps));
        }
      }
#pragma unroll 4
      for (int64_t r = r0 + st; r < r1; r += S) {
        const float4 v = x[r * ldx4 + cg];
        float4 o;
        o.x = norm_elem(v.x, mu[0], den[0], norm, clip);
        o.y = norm_elem(v.y, mu[1], den[1], norm, clip);
        o.z = norm_elem(v.z, mu[2], den[2], norm, clip);
        o.w = norm_elem(v.w, mu[3], den[3], norm, clip);
        bad |= !isfinite(o.x) || !isfinite(o.y) || !isfinite(o.z) || !isfinite(o.w);
        if (y) __stcs(y + r * ldy4 + cg, o);
        if (yb) {
          uint2 packed;
          packed.x = (uint32_t)to_half_bits<FP16>(o.x) | ((uint32_t)to_half_bits<FP16>(o.y) << 16);
          packed.y = (uint32_t)to_half_bits<FP16>(o.z) | ((uint32_t)to_half_bits<FP16>(o.w) << 16);
          yb[r * ldb4 + cg] = packed;
        }
      }
    } else {
      for (int64_t r = r0 + st; r < r1; r += S) yb[r * ldb4 + cg] = make_uint2(0u, 0u);
    }
  }
  if (nonfinite && __any_sync(0xffffffffu, bad) && (threadIdx.x & 31) == 0) atomicAdd(nonfinite, 1u);
}

// Launch of the normalise / cast: the 16-byte kernel when the layout allows it.
inline void launch_apply(const float* x, int64_t B, int D, int64_t ldx, const float* mean, const float* var,
                         float eps, float clip, float* y, int64_t ldy, void* yh, int64_t ldb, bool fp16,
                         unsigned* nonfinite, cudaStream_t s) {
  uint16_t* yb = reinterpret_cast<uint16_t*>(yh);
  const bool vec = D % 4 == 0 && ldx % 4 == 0 && aligned(x, 16) && (!y || (ldy % 4 == 0 && aligned(y, 16))) &&
                   (!yb || (ldb % 4 == 0 && aligned(yb, 8))) && (yb ? ldb / 4 : D / 4) <= NORM_THREADS;
  if (!vec) {
    const unsigned grid = (unsigned)((B + APPLY_ROWS - 1) / APPLY_ROWS);
    if (fp16) k_norm_apply<true><<<grid, NORM_THREADS, 0, s>>>(x, B, D, ldx, mean, var, eps, clip, y, ldy, yb, ldb,
                                                               nonfinite);
    else k_norm_apply<false><<<grid, NORM_THREADS, 0, s>>>(x, B, D, ldx, mean, var, eps, clip, y, ldy, yb, ldb,
                                                           nonfinite);
    return;
  }
  const int64_t slots = (int64_t)sm_count() * APPLY4_BLOCKS_PER_SM * APPLY4_WAVES;
  int64_t rpb = (B + slots - 1) / slots;
  if (rpb < APPLY4_MIN_ROWS) rpb = APPLY4_MIN_ROWS;
  const unsigned grid = (unsigned)((B + rpb - 1) / rpb);
  if (fp16)
    k_norm_apply4<true><<<grid, NORM_THREADS, 0, s>>>(reinterpret_cast<const float4*>(x), B, D, ldx / 4, mean, var,
                                                      eps, clip, reinterpret_cast<float4*>(y), ldy / 4,
                                                      reinterpret_cast<uint2*>(yb), ldb / 4, nonfinite, rpb);
  else
    k_norm_apply4<false><<<grid, NORM_THREADS, 0, s>>>(reinterpret_cast<const float4*>(x), B, D, ldx / 4, mean, var,
                                                       eps, clip, reinterpret_cast<float4*>(y), ldy / 4,
                                                       reinterpret_cast<uint2*>(yb), ldb / 4, nonfinite, rpb);
}

// ---------------------------------------------------------------- rollout bookkeeping
// One thread per environment, the per-step statistics of collect_rollout (ppo_gpu.py:1914-1960)
// in one pass: rollout reward row, next-done flags, running episode return / length, and the
// sums (episode return / length / count, wins, losses, hard-deck losses, opponent hard-deck
// wins, per-opponent wins / losses / episodes).  Per-block sums go to fp64 global accumulators
// with one atomic per block and statistic.
constexpr int REC_THREADS = 256;
constexpr int REC_MAX_OPP = 32;

__global__ void __launch_bounds__(REC_THREADS)
k_rollout_record(int64_t nenv, const double* __restrict__ reward, const uint8_t* __restrict__ done,
                 const double* __restrict__ thp, const double* __restrict__ talt, const int64_t* __restrict__ opp,
                 int n_opp, double min_alt, const uint8_t* __restrict__ finite, float* __restrict__ b_rew,
                 float* __restrict__ next_done, float* __restrict__ ep_ret, float* __restrict__ ep_len,
                 double* __restrict__ stats) {
  __shared__ double red[7][REC_THREADS / 32];
  __shared__ unsigned by_opp[3 * REC_MAX_OPP];
  __shared__ unsigned any_bad;
  for (int i = threadIdx.x; i < 3 * n_opp; i += blockDim.x) by_opp[i] = 0;
  if (threadIdx.x == 0) any_bad = 0;
  __syncthreads();
  int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  double v[7] = {0, 0, 0, 0, 0, 0, 0};
  if (e < nenv) {
    const float r = (float)reward[2 * e];                 // reward[:, 0].float()
    const bool d = done[e] != 0;
    const float df = d ? 1.0f : 0.0f;
    b_rew[e] = r;
    next_done[e] = df;
    const float er = __fadd_rn(ep_ret[e], r);             // ep_ret += raw_reward
    const float el = __fadd_rn(ep_len[e], 1.0f);          // ep_len += 1.0
    v[0] = (double)__fmul_rn(er, df);                     // (ep_ret * done_env).sum()
    v[1] = (double)__fmul_rn(el, df);
    v[2] = (double)df;
    const float keep = __fsub_rn(1.0f, df);
    ep_ret[e] = __fmul_rn(er, keep);
    ep_len[e] = __fmul_rn(el, keep);
    const double th0 = thp[2 * e], th1 = thp[2 * e + 1], ta0 = talt[2 * e], ta1 = talt[2 * e + 1];
    const bool own_alt_dead = ta0 < min_alt;
    const bool own_dead = (th0 <= 0.0) || own_alt_dead;
    const bool opp_dead = (th1 <= 0.0) || (ta1 < min_alt);
    const bool both_alive = !own_dead && !opp_dead;
    const bool win = (opp_dead && !own_dead) || (both_alive && (th0 > th1 + 1e-9));
    const bool loss = (own_dead && !opp_dead) || (both_alive && (th0 < th1 - 1e-9));
    const bool dwin = win && d, dloss = loss && d;
    v[3] = dwin; v[4] = dloss;
    v[5] = loss && own_alt_dead && d;
    v[6] = win && (ta1 < min_alt) && d;
    if (opp) {
      const int64_t g = opp[e];
      if (g >= 0 && g < n_opp) {
        if (dwin) atomicAdd(&by_opp[g], 1u);
        if (dloss) atomicAdd(&by_opp[n_opp + g], 1u);
        if (d) atomicAdd(&by_opp[2 * n_opp + g], 1u);
      }
    }
    if (finite && !finite[e]) atomicOr(&any_bad, 1u);
  }
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
  for (int k = 0; k < 7; k++) {
    double x = v[k];
    for (int o = 16; o > 0; o >>= 1) x += __shfl_xor_sync(0xffffffffu, x, o);
    if (lane == 0) red[k][w] = x;
  }
  __syncthreads();
  if (threadIdx.x < 7) {
    double x = 0.0;
    for (int i = 0; i < REC_THREADS / 32; i++) x += red[threadIdx.x][i];
    if (x != 0.0) atomicAdd(&stats[threadIdx.x], x);
  }
  for (int i = threadIdx.x; i < 3 * n_opp; i += blockDim.x)
    if (by_opp[i]) atomicAdd(&stats[8 + i], (double)by_opp[i]);
  if (threadIdx.x == 0 && any_bad) stats[7] = 1.0;           // trajectory non-finite
}

}  // namespace ro
}  // namespace f16

using namespace f16;

extern "C" int f16_rollout_record(int64_t nenv, const f16_record_args* a, f16_stream_t stream) {
  if (!a || nenv <= 0 || !a->reward || !a->done || !a->terminal_hp || !a->terminal_alt || !a->b_rew ||
      !a->next_done || !a->ep_ret || !a->ep_len || !a->stats)
    return F16_ERR_ARG;
  if (a->n_opp < 0 || a->n_opp > ro::REC_MAX_OPP || (a->opp_row && a->n_opp == 0)) return F16_ERR_ARG;
  int grid = (int)((nenv + ro::REC_THREADS - 1) / ro::REC_THREADS);
  ro::k_rollout_record<<<grid, ro::REC_THREADS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      nenv, a->reward, a->done, a->terminal_hp, a->terminal_alt, a->opp_row, a->n_opp, a->min_alt, a->finite,
      a->b_rew, a->next_done, a->ep_ret, a->ep_len, a->stats);
  return launch_status();
}

namespace f16 {
namespace ro {
// One thread per environment (batched_payoff.py:131-156): first-game scoring of the left policy.
__global__ void __launch_bounds__(256) k_payoff_record(int64_t nenv, const f16_payoff_args a) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nenv || a.finished[e]) return;
  const int ls = a.left_slot[e] ? 1 : 0;
  const double lhp = a.terminal_hp[2 * e + ls], rhp = a.terminal_hp[2 * e + 1 - ls];
  const double lalt = a.terminal_alt[2 * e + ls], ralt = a.terminal_alt[2 * e + 1 - ls];
  const bool ok = a.finite[e] && isfinite(lhp) && isfinite(rhp) && isfinite(lalt) && isfinite(ralt) &&
                  isfinite(a.reward[2 * e]) && isfinite(a.reward[2 * e + 1]);
  if (!ok) atomicAdd(a.nonfinite, 1);
  if (!a.done[e]) return;
  const bool ld = (lhp <= 0.0) || (lalt < a.min_alt);
  const bool rd = (rhp <= 0.0) || (ralt < a.min_alt);
  const bool alive = !ld && !rd;
  const bool win = (rd && !ld) || (alive && (lhp > rhp + 1e-9));
  const bool loss = (ld && !rd) || (alive && (lhp < rhp - 1e-9));
  a.scores[e] = win ? 1.0f : (loss ? 0.0f : 0.5f);
  a.own_crash[e] = lalt < a.min_alt;
  a.opp_crash[e] = ralt < a.min_alt;
  a.finished[e] = 1;
  const int64_t m = e / a.lanes;
  if ((int64_t)atomicAdd(&a.finished_count[m], 1) + 1 == a.lanes)
    a.final_step[m] = a.step + (a.step_dev ? (int32_t)*a.step_dev : 0);
}
}  // namespace ro
}  // namespace f16

extern "C" int f16_payoff_record(int64_t nenv, const f16_payoff_args* a, f16_stream_t stream) {
  if (!a || nenv <= 0 || a->lanes <= 0 || !a->done || !a->terminal_hp || !a->terminal_alt || !a->finite ||
      !a->reward || !a->left_slot || !a->finished || !a->scores || !a->own_crash || !a->opp_crash ||
      !a->finished_count || !a->final_step || !a->nonfinite)
    return F16_ERR_ARG;
  const int grid = (int)((nenv + 255) / 256);
  ro::k_payoff_record<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(nenv, *a);
  return launch_status();
}

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

namespace f16 {
namespace ro {
// The partial-sum pass of the norm update: the 16-byte kernel when the layout allows it.
inline void launch_partial(const float* x, int64_t B, int D, int64_t ldx, double2* part, int64_t nblk,
                           cudaStream_t s) {
  const bool vec = (D % 4 == 0) && (ldx % 4 == 0) && aligned(x, 16) && D / 4 <= PART4_THREADS && D >= 4;
  if (!vec) {
    k_norm_partial<<<(unsigned)nblk, NORM_THREADS, 0, s>>>(x, B, D, ldx, part);
    return;
  }
  const int S = PART4_THREADS / (D / 4);
  const size_t smem = (size_t)S * D * sizeof(double2);
  static bool attr[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr[dev]) {
    cudaFuncSetAttribute(k_norm_partial4, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024);
    attr[dev] = true;
  }
  k_norm_partial4<<<(unsigned)nblk, PART4_THREADS, smem, s>>>(reinterpret_cast<const float4*>(x), B, D, ldx / 4,
                                                               part);
}
}  // namespace ro
}  // namespace f16

extern "C" int f16_norm_update(const float* x, int64_t B, int D, int64_t ldx, float* mean, float* var, float* count,
                               double* scratch, int64_t scratch_doubles, f16_stream_t stream) {
  if (!x || !mean || !var || !count || !scratch || B <= 0 || D <= 0 || ldx < D) return F16_ERR_ARG;
  int nblk = (int)((B + ro::NORM_ROWS_PER_BLOCK - 1) / ro::NORM_ROWS_PER_BLOCK);
  if (scratch_doubles < (int64_t)nblk * D * 2) return F16_ERR_TOO_LARGE;
  if (!aligned(scratch, 16)) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  double2* part = reinterpret_cast<double2*>(scratch);
  ro::launch_partial(x, B, D, ldx, part, nblk, s);
  ro::k_norm_merge<<<(D + 31) / 32, ro::NORM_THREADS, 0, s>>>(part, nblk, B, D,
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
  ro::launch_partial(x, B, D, ldx, part, nblk, s);
  ro::k_norm_reduce<<<(D + 31) / 32, ro::NORM_THREADS, 0, s>>>(
      part, nblk, D, reinterpret_cast<double2*>(sums));
  return launch_status();
}

extern "C" int f16_norm_merge_sums(const double* sums, int64_t B_total, int D, float* mean, float* var,
                                   float* count, f16_stream_t stream) {
  if (!sums || !mean || !var || !count || B_total <= 0 || D <= 0) return F16_ERR_ARG;
  if (!aligned(sums, 16)) return F16_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  ro::k_norm_merge<<<(D + 31) / 32, ro::NORM_THREADS, 0, s>>>(
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
  ro::launch_apply(x, B, D, ldx, mean, var, (float)eps, (float)clip, y, ldy, y_bf16, ldb, false, nullptr,
                   reinterpret_cast<cudaStream_t>(stream));
  return launch_status();
}

extern "C" int f16_norm_apply_checked(const float* x, int64_t B, int D, int64_t ldx, const float* mean,
                                      const float* var, double eps, double clip, float* y, int64_t ldy, void* y_bf16,
                                      int64_t ldb, uint32_t* nonfinite, f16_stream_t stream) {
  if (!x || B <= 0 || D <= 0 || ldx < D || (!y && !y_bf16) || (!mean != !var)) return F16_ERR_ARG;
  if ((y && ldy < D) || (y_bf16 && ldb < D)) return F16_ERR_ARG;
  ro::launch_apply(x, B, D, ldx, mean, var, (float)eps, (float)clip, y, ldy, y_bf16, ldb, false, nonfinite,
                   reinterpret_cast<cudaStream_t>(stream));
  return launch_status();
}

extern "C" int f16_norm_apply_half(const float* x, int64_t B, int D, int64_t ldx, const float* mean,
                                   const float* var, double eps, double clip, float* y, int64_t ldy, void* y_half,
                                   int64_t ldh, int operand, uint32_t* nonfinite, f16_stream_t stream) {
  if (!x || B <= 0 || D <= 0 || ldx < D || (!y && !y_half) || (!mean != !var)) return F16_ERR_ARG;
  if ((y && ldy < D) || (y_half && ldh < D)) return F16_ERR_ARG;
  if (operand != F16_OPERAND_BF16 && operand != F16_OPERAND_FP16) return F16_ERR_ARG;
  ro::launch_apply(x, B, D, ldx, mean, var, (float)eps, (float)clip, y, ldy, y_half, ldh,
                   operand == F16_OPERAND_FP16, nonfinite, reinterpret_cast<cudaStream_t>(stream));
  return launch_status();
}

namespace f16 {
namespace ro {
// One warp per input row: the row's group picks its normaliser (or none), the 16-bit result goes
// to the row's destination in the grouped, tile-aligned policy input.
template <bool FP16>
__global__ void __launch_bounds__(NORM_THREADS)
k_norm_apply_scatter(const float* __restrict__ x, int64_t B, int D, int64_t ldx, const int64_t* __restrict__ grp,
                     const int64_t* __restrict__ dst, const float* const* __restrict__ means,
                     const float* const* __restrict__ vars, int n_groups, float eps, float clip,
                     uint16_t* __restrict__ y, int64_t ldh, unsigned* __restrict__ nonfinite) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * (NORM_THREADS / 32) + (threadIdx.x >> 5);
  if (r >= B) return;
  const int64_t g = grp[r];
  if (g < 0 || g >= n_groups) {
    if (lane == 0 && nonfinite) atomicOr(nonfinite, 0x80000000u);
    return;
  }
  const float* mu = means[g];
  const float* va = vars[g];
  const bool norm = mu != nullptr && va != nullptr;
  uint16_t* out = y + dst[r] * ldh;
  bool bad = false;
  for (int d = lane; d < ldh; d += 32) {
    if (d < D) {
      float o = x[r * ldx + d];
      if (norm) {
        o = __fdiv_rn(__fsub_rn(o, mu[d]), __fsqrt_rn(__fadd_rn(va[d], eps)));
        o = o < -clip ? -clip : (o > clip ? clip : o);
      }
      bad |= !isfinite(o);
      out[d] = to_half_bits<FP16>(o);
    } else {
      out[d] = 0;
    }
  }
  if (nonfinite && __any_sync(0xffffffffu, bad) && lane == 0) atomicAdd(nonfinite, 1u);
}
}  // namespace ro
}  // namespace f16

extern "C" int f16_norm_apply_scatter(const float* x, int64_t B, int D, int64_t ldx, const int64_t* group_of_row,
                                      const int64_t* dst_row, const float* const* mean_ptrs,
                                      const float* const* var_ptrs, int n_groups, double eps, double clip,
                                      void* y_half, int64_t ldh, int operand, uint32_t* nonfinite,
                                      f16_stream_t stream) {
  if (!x || !group_of_row || !dst_row || !mean_ptrs || !var_ptrs || !y_half || B < 0 || D <= 0 || ldx < D ||
      ldh < D || n_groups < 1)
    return F16_ERR_ARG;
  if (operand != F16_OPERAND_BF16 && operand != F16_OPERAND_FP16) return F16_ERR_ARG;
  if (B == 0) return F16_OK;
  const unsigned grid = (unsigned)((B + ro::NORM_THREADS / 32 - 1) / (ro::NORM_THREADS / 32));
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  uint16_t* y = reinterpret_cast<uint16_t*>(y_half);
  if (operand == F16_OPERAND_FP16)
    ro::k_norm_apply_scatter<true><<<grid, ro::NORM_THREADS, 0, s>>>(x, B, D, ldx, group_of_row, dst_row, mean_ptrs,
                                                                     var_ptrs, n_groups, (float)eps, (float)clip, y,
                                                                     ldh, nonfinite);
  else
    ro::k_norm_apply_scatter<false><<<grid, ro::NORM_THREADS, 0, s>>>(x, B, D, ldx, group_of_row, dst_row, mean_ptrs,
                                                                      var_ptrs, n_groups, (float)eps, (float)clip, y,
                                                                      ldh, nonfinite);
  return launch_status();
}

// ---------------------------------------------------------------------------------------------
// RunningNorm update with library-owned scratch (no counterpart in the reference).
//
// For callers that cannot allocate device memory at the point of the update: a fixed-size
// memory pool or arena that is sealed once training starts, or a host driver that forbids
// allocation inside its step loop.  The fp64 partial sums live in a file-scope device array of
// F16_NORM_STATIC_SCRATCH_PAIRS double2 (2 MiB) instead of a caller buffer; its device address
// comes from cudaGetSymbolAddress with the device current: looked up again on every call made
// outside a stream capture (so a device reset between calls leaves no stale address), and the
// last address found is used inside a capture.  Every scratch slot that the merge kernel reads is
// written by the partial kernel of the same call first, so nothing needs to start at zero.
// There is one array per device, so two calls in flight at the same time on one device (two
// streams, or two host threads) race on it; calls queued on one stream are ordered and safe.
// ---------------------------------------------------------------------------------------------
static __device__ __align__(256) double2 g_norm_static_scratch[F16_NORM_STATIC_SCRATCH_PAIRS];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_norm_static_mu;
double2* g_norm_static_addr[kMaxDevices] = {};

// Device address of g_norm_static_scratch on the current device: looked up whenever `s` is not
// capturing, the cached one while it is.
int norm_static_scratch(cudaStream_t s, double2** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return F16_ERR_CUDA;
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cs) != cudaSuccess) {
    cudaGetLastError();
    return F16_ERR_CUDA;
  }
  std::lock_guard<std::mutex> lock(g_norm_static_mu);
  if (cs == cudaStreamCaptureStatusNone || !g_norm_static_addr[dev]) {
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
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  double2* part = nullptr;
  int rc = norm_static_scratch(s, &part);
  if (rc != F16_OK) return rc;
  ro::launch_partial(x, B, D, ldx, part, nblk, s);
  ro::k_norm_merge<<<(D + 31) / 32, ro::NORM_THREADS, 0, s>>>(
      part, (int)nblk, B, D, mean, var, count);
  ro::k_norm_count<<<1, 32, 0, s>>>(count, B);
  return launch_status();
}
