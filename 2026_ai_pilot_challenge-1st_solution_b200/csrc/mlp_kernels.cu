// mlp_kernels.cu -- policy / value MLP forward on the 5th-generation tensor cores (sm_100a).
//
// Replaces the rollout-time forwards of R/claude_code/model.py MLPDiscreteActorCritic
// (actor_logits / critic, :162-241) as driven by ppo_gpu.py actor_step / value_step (:273-291)
// and the frozen-opponent pools (:536-592, :877-898), including the Categorical sample and its
// summed log-probability (inverse-CDF sampling on the softmax weights, fused into the last layer's
// epilogue).
//
// One persistent CTA per SM processes "jobs" = (128-row tile, network).  Per job and layer:
//   * the A operand (the 128 x K activation tile, 16-bit: bf16 or fp16, one type per network set)
//     lives in a 128 KB shared-memory region in
//     the K-major 128-byte-swizzled layout the tensor core reads; layer 0's A is loaded by TMA,
//     layer l's A is written there by layer l-1's epilogue;
//   * weight tiles (nn.Linear layout = K-major B) stream through a 3-stage ring of 32 KB TMA
//     boxes (256 output rows x 64 inputs), each CTA loading its own copy;
//   * one thread issues tcgen05.mma (M=128, N<=256, K=16 per instruction) accumulating fp32 in
//     TMEM (all 512 columns = a full 128 x 512 layer);
//   * four epilogue warps tcgen05.ld their 32 TMEM lanes, add bias, apply ReLU/tanh, and write the
//     16-bit activations back to shared memory (or run the output head).
// Operand type: bf16 (8-bit significand) or fp16 (11-bit significand, same tensor throughput).
// Against the fp32 network fp16 operands cut the logit error about eightfold (round-off 2^-11
// instead of 2^-8 per input, weight and hidden activation), which brings logits and log-probs
// within 1e-3 of fp32; fp16 hidden activations are converted with saturation (+-65504), so an
// out-of-range activation clamps instead of becoming infinite.
// Every mbarrier wait is bounded by a clock deadline; a timeout sets an error code and all roles
// leave their loops, so a malformed launch returns an error instead of hanging.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>
#include "common.cuh"

namespace f16 {
namespace mlp {

constexpr int MAX_LAYERS = 4;
constexpr int MAX_NETS = 20;
constexpr int TILE_M = 128;
constexpr int KCHUNK = 64;                       // bf16 elements per 128-byte swizzle row
constexpr int NCHUNK = 256;                      // output columns per MMA / weight box
constexpr int STAGES = 3;
constexpr int ACT_BYTES = 128 * 1024;            // 8 chunks x (128 rows x 128 B)
constexpr int STAGE_BYTES = NCHUNK * 128;        // 32 KB
// Four epilogue warps per quarter (18 warps, 96 registers): with the split hidden layers each
// thread holds two packed chunks of the first half; measured 0.326 ms for the rollout's actor +
// critic launch against 0.335 ms for two warps without the split and 0.367 ms for two warps
// with it (register spills).
#ifndef F16_MLP_EPI_PER_QUARTER
#define F16_MLP_EPI_PER_QUARTER 4
#endif
constexpr int EPI_PER_Q = F16_MLP_EPI_PER_QUARTER;   // epilogue warps per TMEM lane quarter (2 or 4)
constexpr int CTRL_BYTES = 2048;                 // barriers, TMEM base, the heads' per-part partials
constexpr int SMEM_BYTES = ACT_BYTES + STAGES * STAGE_BYTES + CTRL_BYTES + 1024;
constexpr int EPI_WARPS = 4 * EPI_PER_Q;         // the warps of a quarter split the columns
constexpr int THREADS = 64 + 32 * EPI_WARPS;     // warp 0 TMA, warp 1 MMA + TMEM, then the epilogue
static_assert(SMEM_BYTES <= 232448, "shared memory per CTA");
constexpr long long WAIT_CYCLES = 4000000000LL;  // ~2 s at 1.9 GHz

enum Head : int { HEAD_HIDDEN_ONLY = 0, HEAD_CATEGORICAL = 1, HEAD_VALUE = 2 };

struct NetDev {
  CUtensorMap w[MAX_LAYERS];                     // weight maps (64-byte aligned, in global memory)
};

struct NetParams {
  const float* bias[MAX_LAYERS];
  int n_layers;
  int in_pad;                                    // K of layer 0 rounded up to 64
  int width[MAX_LAYERS];                         // true output width of each layer
  int width_pad[MAX_LAYERS];                     // hidden: multiple of 64; last: multiple of 16
  int act;                                       // 0 relu, 1 tanh
  int head;                                      // Head
  int num_bins, act_dim;                         // categorical head: act_dim groups of num_bins
  int fp16;                                      // operands: 0 bf16, 1 fp16 (one type per set)
  // A width-1 value head after at least one hidden layer is not run on the tensor cores: the
  // last hidden layer's epilogue keeps its activations in fp32 and dots them with the head's
  // weight row (head_w32 when given, else the 16-bit row head_w16 converted), so the head needs
  // no MMA, no 16-bit activation tile and no extra pass over TMEM.
  int fold;
  const float* head_w32;
  const void* head_w16;
};

// Every network's parameters travel in the kernel's parameter space (constant bank): each role
// reads the current job's fields there with uniform, cached loads instead of global-memory
// loads whose latency sat between a job's layers.
struct NetTable {
  NetParams p[MAX_NETS];
};

struct Launch {
  int64_t rows;                                  // valid rows of X
  int n_groups;                                  // row groups (frozen-opponent pools); group g owns
  int64_t group_end[MAX_NETS + 1];               //   rows [group_end[g-1], group_end[g]); starts % 128 == 0
  const int64_t* group_end_dev;                  // the same ends read from device memory instead (a
                                                 //   grouping computed on the device); tiles_total is
                                                 //   then an upper bound and surplus jobs are skipped
  int group_net[MAX_NETS][2];                    // networks per group (second = -1 if none)
  int nets_per_group;
  int64_t tiles_total;                           // sum over groups of ceil(rows_g / 128)
  // outputs (row index = X row)
  uint8_t* bins; int64_t bins_stride; int bins_offset;   // sampled action bins (act_dim bytes per row)
  int32_t* act_idx;                              // optional int32 [rows][act_dim]
  float* logp;                                   // summed log-probability per row
  float* value;                                  // value head output per row
  float* logits; int64_t logits_ld;              // optional raw logits / value (tests)
  uint64_t seed, step;
  const uint64_t* step_dev;                      // optional device counter added to step
  int deterministic;                             // argmax instead of sampling
  int* err;
  double* cmd; int64_t cmd_stride; int cmd_offset;   // optional env commands of the bins
  const float* grid;                             //   (fp32 action grid, num_bins values)
};

// ---------------------------------------------------------------- PTX helpers
__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait: false on timeout or when another role already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (*abort_flag) return false;
    if (clock64() - t0 > WAIT_CYCLES) {
      *abort_flag = 1;
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// 32 consecutive fp32 columns of this warp's 32 TMEM lanes, without the completion wait
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// 8 consecutive fp32 columns of this warp's 32 TMEM lanes, without the completion wait
__device__ __forceinline__ void tmem_ld8_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 16 packed 32-bit words of this warp's 32 TMEM lanes: store / load (load waits for completion)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint4 (&w)[4]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(w[0].x), "r"(w[0].y), "r"(w[0].z), "r"(w[0].w), "r"(w[1].x), "r"(w[1].y), "r"(w[1].z),
        "r"(w[1].w), "r"(w[2].x), "r"(w[2].y), "r"(w[2].z), "r"(w[2].w), "r"(w[3].x), "r"(w[3].y), "r"(w[3].z),
        "r"(w[3].w)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint4 (&w)[4]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(w[0].x), "=r"(w[0].y), "=r"(w[0].z), "=r"(w[0].w), "=r"(w[1].x), "=r"(w[1].y), "=r"(w[1].z),
        "=r"(w[1].w), "=r"(w[2].x), "=r"(w[2].y), "=r"(w[2].z), "=r"(w[2].w), "=r"(w[3].x), "=r"(w[3].y),
        "=r"(w[3].z), "=r"(w[3].w)
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// K-major, 128-byte-swizzled shared-memory matrix descriptor (rows 128 B apart in groups of 8,
// groups 1024 B apart): start>>4 | LBO 16 B | SBO 1024 B | version 1 | layout SWIZZLE_128B.
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// kind::f16 instruction descriptor: fp32 accumulate, A and B both bf16 (format 1) or both fp16
// (format 0), both K-major, M = 128.
template <bool FP16>
__device__ __forceinline__ uint32_t idesc_f16(int n) {
  const uint32_t ab = FP16 ? 0u : ((1u << 7) | (1u << 10));
  return (1u << 4) | ab | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// ---------------------------------------------------------------- job decoding
struct Job {
  int64_t row0;
  int rows;
  int net;
};
// A hidden layer two weight boxes wide (512 outputs): the MMA issuer signals its first 256
// accumulator columns (acc_h0) before issuing the second half, and the epilogue converts that
// half while the second half's MMAs run, parking the packed 16-bit values in the columns it has
// read; it stores them to shared memory once the layer's MMAs are done reading the activations
// they replace (acc_full).
__device__ __forceinline__ bool split_layer(const NetParams& P, int l) {
  return l < P.n_layers - 1 && P.width_pad[l] == 2 * NCHUNK;
}

// K-chunks per ring stage of a layer: a layer at most 128 outputs wide moves boxes of at most
// 128 rows, so several K-chunks share one 32 KB stage (the output head's weights then arrive in
// one or a few stages, mostly prefetched while the previous layer runs); wider layers move one
// 256-row box per stage.
__device__ __forceinline__ int chunks_per_stage(int N, int K) {
  const int rows = N < NCHUNK ? N : NCHUNK;
  if (rows > NCHUNK / 2) return 1;
  const int c = NCHUNK / rows, kc = K / KCHUNK;
  return c < kc ? c : kc;
}

__device__ __forceinline__ bool decode_job(const Launch& L, int64_t j, Job& J) {
  int64_t tile = j / L.nets_per_group;
  int slot = (int)(j % L.nets_per_group);
  // CTA b runs jobs b, b + G, b + 2G, ...: with two networks per group and an even grid G every
  // job of a CTA would have b's parity (the same network); swapping the two networks on
  // alternate rounds gives each CTA both (jobs 2t, 2t+1 share a round, so this stays a
  // one-to-one map of jobs)
  if (L.nets_per_group == 2 && (gridDim.x & 1) == 0) slot ^= (int)((j / gridDim.x) & 1);
  int64_t start = 0;
  for (int g = 0; g < L.n_groups; g++) {
    int64_t end = L.group_end_dev ? __ldg(L.group_end_dev + g) : L.group_end[g];
    end = end < L.rows ? end : L.rows;           // never past the input rows
    end = end > start ? end : start;             // an empty (or malformed) group has no tiles
    int64_t nt = (end - start + TILE_M - 1) / TILE_M;
    if (tile < nt) {
      J.row0 = start + tile * TILE_M;
      int64_t r = end - J.row0;
      J.rows = (int)(r < TILE_M ? r : TILE_M);
      J.net = L.group_net[g][slot];
      return J.net >= 0;
    }
    tile -= nt;
    start = end;
  }
  return false;
}

__device__ __forceinline__ uint64_t mix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
// Sampling noise: a 64-bit key per (call, row) from splitmix64, then per channel a 32-bit
// avalanche mix (Wellons' "lowbias32" constants) of the key and the channel index, giving a
// 24-bit uniform u in (0,1).  The channel's bin is the first whose running sum of the softmax
// weights exp(x - max) exceeds u times their total: inverse-CDF sampling, one uniform per
// channel, reusing the exponentials of the log-sum-exp.
__device__ __forceinline__ uint64_t row_key(uint64_t seed, uint64_t step, int64_t row) {
  return mix64(seed ^ mix64((step << 32) ^ ((uint64_t)row * 0x9E3779B97F4A7C15ull)));
}
__device__ __forceinline__ float uniform24(uint64_t key, uint32_t idx) {
  uint32_t x = ((uint32_t)key ^ (idx * 0x9E3779B9u)) + (uint32_t)(key >> 32);
  x ^= x >> 16;
  x *= 0x7feb352du;
  x ^= x >> 15;
  x *= 0x846ca68bu;
  x ^= x >> 16;
  return ((float)(x >> 8) + 0.5f) * (1.0f / 16777216.0f);
}

struct Smem {
  uint64_t x_full, act_empty, acc_full, act_ready, tmem_empty, drain, logp_bar;
  uint64_t act_lo;                               // a 512-wide layer's first 256 activations stored
  uint64_t acc_h0;                               // a 512-wide hidden layer's first 256 columns done
  uint64_t full[STAGES], empty[STAGES];
  uint32_t tmem_base;
  int abort_flag;
  float logp_part[EPI_PER_Q - 1][TILE_M];        // the other parts' log-probs (or value partial sums) per row
};
static_assert(sizeof(Smem) <= CTRL_BYTES, "control block");
static_assert(sizeof(NetTable) + sizeof(Launch) + sizeof(CUtensorMap) + sizeof(void*) <= 4096, "kernel parameters");

// tanh for hidden activations that are rounded to bf16 right after: the hardware approximation
// (max relative error about 2^-11) is well below the bf16 rounding step (2^-9).
__device__ __forceinline__ float tanh_fast(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// two fp32 lanes at once (Blackwell packed f32x2 add, round to nearest like a scalar add)
__device__ __forceinline__ uint64_t add_f32x2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
// pack two fp32 (lo, hi) into bf16x2 or fp16x2 with round-to-nearest, optionally clamping at 0
// first (relu(round(x)) == round(relu(x)), so the fused clamp gives the same bits as relu then
// round); fp16 saturates at +-65504 (NaN stays NaN)
template <bool FP16>
__device__ __forceinline__ uint32_t pack_x2(uint64_t v, bool relu) {
  const float lo = __uint_as_float((uint32_t)v), hi = __uint_as_float((uint32_t)(v >> 32));
  uint32_t d;
  if (FP16) {
    if (relu) asm("cvt.rn.relu.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    else asm("cvt.rn.satfinite.f16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  } else {
    if (relu) asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    else asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
  }
  return d;
}

// bias + activation of 32 accumulator columns [c0, c0+32) of one row, packed to bf16 into the
// row's 128-byte swizzled line of the next layer's A operand: all bias loads first (one exposed
// latency per chunk), the bias added two lanes per instruction, one activation branch per chunk,
// ReLU fused into the conversion
// bias + activation of one 32-column chunk packed as the four 16-byte units it stores
template <bool FP16>
__device__ __forceinline__ void pack32(const uint32_t (&r)[32], const ulonglong2 (&bv)[8], bool relu,
                                       uint4 (&w)[4]) {
  uint64_t x[16];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    x[2 * i] = add_f32x2(((uint64_t)r[4 * i + 1] << 32) | r[4 * i], bv[i].x);
    x[2 * i + 1] = add_f32x2(((uint64_t)r[4 * i + 3] << 32) | r[4 * i + 2], bv[i].y);
  }
  if (!relu) {
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float lo = tanh_fast(__uint_as_float((uint32_t)x[i]));
      const float hi = tanh_fast(__uint_as_float((uint32_t)(x[i] >> 32)));
      x[i] = ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
    }
  }
#pragma unroll
  for (int u = 0; u < 4; u++) {
    w[u].x = pack_x2<FP16>(x[4 * u + 0], relu);
    w[u].y = pack_x2<FP16>(x[4 * u + 1], relu);
    w[u].z = pack_x2<FP16>(x[4 * u + 2], relu);
    w[u].w = pack_x2<FP16>(x[4 * u + 3], relu);
  }
}
// the 32 biases of a chunk, loaded before its TMEM load so that the two latencies overlap
__device__ __forceinline__ void load_bias32(const float* __restrict__ bias, int c0, ulonglong2 (&bv)[8]) {
  const ulonglong2* b2 = reinterpret_cast<const ulonglong2*>(bias + c0);
#pragma unroll
  for (int i = 0; i < 8; i++) bv[i] = __ldg(b2 + i);
}
// the packed chunk into the swizzled A region of the next layer (row m, columns c0..c0+31)
__device__ __forceinline__ void store32(const uint4 (&w)[4], uint8_t* rowbase, int c0, int m) {
  uint8_t* rowp = rowbase + (c0 / KCHUNK) * TILE_M * 128;
  const int unit0 = (c0 % KCHUNK) / 8;
#pragma unroll
  for (int u = 0; u < 4; u++) *reinterpret_cast<uint4*>(rowp + (((unit0 + u) ^ (m & 7)) * 16)) = w[u];
}

template <bool FP16>
__device__ __forceinline__ void convert32(const uint32_t (&r)[32], const ulonglong2 (&bv)[8], int c0, uint8_t* rowbase,
                                          int m, bool relu) {
  uint64_t x[16];
#pragma unroll
  for (int i = 0; i < 8; i++) {
    x[2 * i] = add_f32x2(((uint64_t)r[4 * i + 1] << 32) | r[4 * i], bv[i].x);
    x[2 * i + 1] = add_f32x2(((uint64_t)r[4 * i + 3] << 32) | r[4 * i + 2], bv[i].y);
  }
  if (!relu) {
#pragma unroll
    for (int i = 0; i < 16; i++) {
      const float lo = tanh_fast(__uint_as_float((uint32_t)x[i]));
      const float hi = tanh_fast(__uint_as_float((uint32_t)(x[i] >> 32)));
      x[i] = ((uint64_t)__float_as_uint(hi) << 32) | __float_as_uint(lo);
    }
  }
  uint8_t* rowp = rowbase + (c0 / KCHUNK) * TILE_M * 128;
  const int unit0 = (c0 % KCHUNK) / 8;
#pragma unroll
  for (int u = 0; u < 4; u++) {                    // 16-byte unit = 8 columns
    uint4 w;
    w.x = pack_x2<FP16>(x[4 * u + 0], relu);
    w.y = pack_x2<FP16>(x[4 * u + 1], relu);
    w.z = pack_x2<FP16>(x[4 * u + 2], relu);
    w.w = pack_x2<FP16>(x[4 * u + 3], relu);
    *reinterpret_cast<uint4*>(rowp + (((unit0 + u) ^ (m & 7)) * 16)) = w;
  }
}

// Folded value head over 16 columns [c0, c0+16) of one row: the biases and head weights (fp32
// row, or the 16-bit row widened) are loaded before the columns' TMEM load so the latencies
// overlap; then bias + activation in fp32 (ReLU keeps NaN, as torch's does; tanh is the accurate
// tanhf, since nothing here is rounded to 16 bits) and the dot product accumulated onto `acc` in
// column order.
struct Fold16 {
  float4 b[4], w[4];
};
template <bool FP16>
__device__ __forceinline__ void fold16_load(const float* __restrict__ bias, const NetParams& P, int c0, Fold16& f) {
  const float4* b4 = reinterpret_cast<const float4*>(bias + c0);
#pragma unroll
  for (int i = 0; i < 4; i++) f.b[i] = __ldg(b4 + i);
  if (P.head_w32) {
    const float4* w4 = reinterpret_cast<const float4*>(P.head_w32 + c0);
#pragma unroll
    for (int i = 0; i < 4; i++) f.w[i] = __ldg(w4 + i);
  } else {
    const uint2* h2 = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(P.head_w16) + c0);
#pragma unroll
    for (int i = 0; i < 4; i++) {
      const uint2 t = __ldg(h2 + i);
      const unsigned short e[4] = {(unsigned short)(t.x & 0xFFFFu), (unsigned short)(t.x >> 16),
                                   (unsigned short)(t.y & 0xFFFFu), (unsigned short)(t.y >> 16)};
      float v[4];
#pragma unroll
      for (int k = 0; k < 4; k++) v[k] = FP16 ? __half2float(__ushort_as_half(e[k])) : __uint_as_float((uint32_t)e[k] << 16);
      f.w[i] = make_float4(v[0], v[1], v[2], v[3]);
    }
  }
}
template <bool RELU>
__device__ __forceinline__ float fold16(const uint4 (&q)[4], const Fold16& f, float acc) {
  const uint32_t r[16] = {q[0].x, q[0].y, q[0].z, q[0].w, q[1].x, q[1].y, q[1].z, q[1].w,
                          q[2].x, q[2].y, q[2].z, q[2].w, q[3].x, q[3].y, q[3].z, q[3].w};
  float h[16];
#pragma unroll
  for (int i = 0; i < 4; i++) {
    h[4 * i] = __uint_as_float(r[4 * i]) + f.b[i].x;
    h[4 * i + 1] = __uint_as_float(r[4 * i + 1]) + f.b[i].y;
    h[4 * i + 2] = __uint_as_float(r[4 * i + 2]) + f.b[i].z;
    h[4 * i + 3] = __uint_as_float(r[4 * i + 3]) + f.b[i].w;
  }
#pragma unroll
  for (int i = 0; i < 16; i++) h[i] = RELU ? (h[i] < 0.0f ? 0.0f : h[i]) : tanhf(h[i]);
#pragma unroll
  for (int i = 0; i < 4; i++) {
    acc = fmaf(h[4 * i], f.w[i].x, acc); acc = fmaf(h[4 * i + 1], f.w[i].y, acc);
    acc = fmaf(h[4 * i + 2], f.w[i].z, acc); acc = fmaf(h[4 * i + 3], f.w[i].w, acc);
  }
  return acc;
}

// The folded head over this warp's chunks c0, c0 + step, ... below c_end, in 16-column steps.
// The activation is a template parameter: a runtime select would issue the tanhf code for ReLU
// networks as well.
template <bool FP16, bool RELU>
__device__ __forceinline__ float fold_chunks(uint32_t lane_addr, uint32_t side, const float* __restrict__ bias,
                                             const NetParams& P, int c0, int c_end, int step, float part) {
  for (int c = c0; c < c_end; c += step) {
#pragma unroll
    for (int k = 0; k < 32; k += 16) {
      uint4 ra[4];
      Fold16 f;
      fold16_load<FP16>(bias, P, c + k, f);
      tmem_ld16(lane_addr + ((uint32_t)(c + k) ^ side), ra);
      part = fold16<RELU>(ra, f, part);
    }
  }
  return part;
}

// Per-row outputs of one sampled channel: bins / int32 index / fp64 env command.
// gv: the action grid's value at `best` (read only when env commands are written).
__device__ __forceinline__ void emit_choice(const Launch& L, int act_dim, int64_t row, int g, int best, float gv) {
  if (L.bins) L.bins[row * L.bins_stride + L.bins_offset + g] = (uint8_t)best;
  if (L.act_idx) L.act_idx[row * act_dim + g] = best;
  if (L.cmd) {
    // action_to_env in fp32: grid value, throttle (channel 3) 0.5 * v + 0.5
    const float cv = g == 3 ? __fadd_rn(__fmul_rn(0.5f, gv), 0.5f) : gv;
    L.cmd[row * L.cmd_stride + L.cmd_offset + g] = (double)cv;
  }
}
__device__ __forceinline__ void emit_choice(const Launch& L, int act_dim, int64_t row, int g, int best) {
  emit_choice(L, act_dim, row, g, best, L.cmd ? __ldg(L.grid + best) : 0.0f);
}

// Categorical head with compile-time shape (the reference's 4 channels x 21 bins), split over
// the PARTS epilogue warps of a lane quarter: part H handles channels [H*A/PARTS, (H+1)*A/PARTS).
// Logits stay in registers; per channel max, log-sum-exp, inverse-CDF sample (or argmax);
// returns this part's share of the summed log-prob.
// grid_lane: this lane's entry of the action grid (lane < NB), so the chosen bin's value comes
// by one warp shuffle instead of a dependent load.
template <int A, int NB, int H, int PARTS>
__device__ __forceinline__ float cat_head(uint32_t lane_addr, const float* __restrict__ bias, const Launch& L,
                                          int64_t row, bool valid, float grid_lane) {
  static_assert(A % PARTS == 0, "channels split evenly over the parts");
  constexpr int GA = A / PARTS;                  // channels of this part
  constexpr int W = GA * NB;
  constexpr int C0 = H * W;                      // first logit column of this half
  constexpr int LB = C0 / 8 * 8;                 // first TMEM column loaded (8-column blocks)
  constexpr int NL = (C0 + W - 1) / 8 - C0 / 8 + 1;
  // the row's sampling key and the biases before the TMEM loads
  const uint64_t key = L.deterministic ? 0ull : row_key(L.seed, L.step + (L.step_dev ? *L.step_dev : 0ull), row);
  float lg[W];
#pragma unroll
  for (int i = 0; i < W; i++) lg[i] = __ldg(bias + C0 + i);
  uint32_t r[NL * 8];
#pragma unroll
  for (int c = 0; c < NL; c++) tmem_ld8_nowait(lane_addr + (uint32_t)(LB + 8 * c), r + 8 * c);
  tmem_wait_ld();
#pragma unroll
  for (int i = 0; i < W; i++) lg[i] += __uint_as_float(r[C0 - LB + i]);
  float logp = 0.0f;
#pragma unroll
  for (int gl = 0; gl < GA; gl++) {
    const int g = H * GA + gl;
    const float* x = lg + gl * NB;
    float mx = x[0];
#pragma unroll
    for (int b = 1; b < NB; b++) mx = fmaxf(mx, x[b]);
    float ex[NB];
    float se = 0.0f;
#pragma unroll
    for (int b = 0; b < NB; b++) {
      ex[b] = __expf(x[b] - mx);
      se += ex[b];
    }
    const float lse = mx + logf(se);
    int best = 0;
    if (L.deterministic) {
      float bestv = -INFINITY;
#pragma unroll
      for (int b = 0; b < NB; b++)
        if (x[b] > bestv) { bestv = x[b]; best = b; }
    } else {
      // the first bin whose running weight exceeds u * total = the number of bins whose running
      // weight does not (running sums never decrease); the last bin if rounding leaves none
      const float target = uniform24(key, (uint32_t)(g * 64)) * se;
      float cum = 0.0f;
      int below = 0;
#pragma unroll
      for (int b = 0; b < NB; b++) {
        cum += ex[b];
        below += cum <= target ? 1 : 0;
      }
      best = below < NB - 1 ? below : NB - 1;
    }
    float chosen = x[0];
#pragma unroll
    for (int b = 1; b < NB; b++) chosen = (b == best) ? x[b] : chosen;
    logp += chosen - lse;
    const float gv = __shfl_sync(0xffffffffu, grid_lane, best);
    if (valid) emit_choice(L, A, row, g, best, gv);
  }
  if (valid && L.logits)
#pragma unroll
    for (int i = 0; i < W; i++) L.logits[row * L.logits_ld + C0 + i] = lg[i];
  return logp;
}

// One channel of NB bins per part (the reference's 4 x 21 shape with four parts per quarter): the
// same code for every part, the channel g a runtime value.  Each part's 21 logit columns start
// at a column offset 21g whose position inside an 8-column block (21g mod 8: 0, 5, 2, 7) picks
// one of four unrolled extractions; everything after them is a single instance.  (A separate
// instance per part put four copies of the head on every scheduler's instruction stream.)
template <int NB, int OFF>
__device__ __forceinline__ void head_extract(const uint32_t (&r)[32], float (&lg)[NB]) {
#pragma unroll
  for (int i = 0; i < NB; i++) lg[i] += __uint_as_float(r[OFF + i]);
}
template <int A, int NB>
__device__ __forceinline__ float cat_head1(uint32_t lane_addr, const float* __restrict__ bias, const Launch& L,
                                           int64_t row, bool valid, float grid_lane, int g) {
  static_assert(NB + 7 <= 32, "a channel's logits fit the four loaded 8-column blocks");
  const int C0 = g * NB, LB = C0 & ~7, off = C0 - LB;
  const uint64_t key = L.deterministic ? 0ull : row_key(L.seed, L.step + (L.step_dev ? *L.step_dev : 0ull), row);
  float x[NB];
#pragma unroll
  for (int i = 0; i < NB; i++) x[i] = __ldg(bias + C0 + i);
  uint32_t r[32];
#pragma unroll
  for (int c = 0; c < 4; c++) tmem_ld8_nowait(lane_addr + (uint32_t)(LB + 8 * c), r + 8 * c);
  tmem_wait_ld();
  switch (off) {
    case 0: head_extract<NB, 0>(r, x); break;
    case 2: head_extract<NB, 2>(r, x); break;
    case 5: head_extract<NB, 5>(r, x); break;
    default: head_extract<NB, 7>(r, x); break;
  }
  float mx = x[0];
#pragma unroll
  for (int b = 1; b < NB; b++) mx = fmaxf(mx, x[b]);
  float ex[NB];
  float se = 0.0f;
#pragma unroll
  for (int b = 0; b < NB; b++) {
    ex[b] = __expf(x[b] - mx);
    se += ex[b];
  }
  const float lse = mx + logf(se);
  int best = 0;
  if (L.deterministic) {
    float bestv = -INFINITY;
#pragma unroll
    for (int b = 0; b < NB; b++)
      if (x[b] > bestv) { bestv = x[b]; best = b; }
  } else {
    // the first bin whose running weight exceeds u * total = the number of bins whose running
    // weight does not (running sums never decrease); the last bin if rounding leaves none
    const float target = uniform24(key, (uint32_t)(g * 64)) * se;
    float cum = 0.0f;
    int below = 0;
#pragma unroll
    for (int b = 0; b < NB; b++) {
      cum += ex[b];
      below += cum <= target ? 1 : 0;
    }
    best = below < NB - 1 ? below : NB - 1;
  }
  float chosen = x[0];
#pragma unroll
  for (int b = 1; b < NB; b++) chosen = (b == best) ? x[b] : chosen;
  const float gv = __shfl_sync(0xffffffffu, grid_lane, best);
  if (valid) emit_choice(L, A, row, g, best, gv);
  if (valid && L.logits)
#pragma unroll
    for (int i = 0; i < NB; i++) L.logits[row * L.logits_ld + C0 + i] = x[i];
  return chosen - lse;
}

// One fp32 column of this warp's 32 TMEM lanes.
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
  return __uint_as_float(r);
}

// Any other categorical shape (act_dim * num_bins <= 96): the logits are re-read from TMEM one
// column at a time in each pass, so no per-thread array (and no local memory) is needed.
__device__ __noinline__ void cat_head_generic(uint32_t lane_addr, const float* __restrict__ bias, const Launch& L,
                                              const NetParams& P, int64_t row, bool valid) {
  const int nb = P.num_bins;
  const uint64_t key = L.deterministic ? 0ull : row_key(L.seed, L.step + (L.step_dev ? *L.step_dev : 0ull), row);
  float logp = 0.0f;
  for (int g = 0; g < P.act_dim; g++) {
    const int c0 = g * nb;
    float mx = -INFINITY;
    for (int b = 0; b < nb; b++) mx = fmaxf(mx, tmem_ld1(lane_addr + (uint32_t)(c0 + b)) + __ldg(bias + c0 + b));
    float se = 0.0f;
    int best = 0;
    float bestv = -INFINITY;
    for (int b = 0; b < nb; b++) {
      const float x = tmem_ld1(lane_addr + (uint32_t)(c0 + b)) + __ldg(bias + c0 + b);
      se += __expf(x - mx);
      if (x > bestv) { bestv = x; best = b; }
      if (valid && L.logits) L.logits[row * L.logits_ld + c0 + b] = x;
    }
    float chosen = bestv;
    if (!L.deterministic) {
      // inverse-CDF sample as in cat_head (a second pass over the channel's logits; every TMEM
      // load reads the same column across the warp, the choice is kept per thread)
      const float target = uniform24(key, (uint32_t)(g * 64)) * se;
      float cum = 0.0f;
      bool found = false;
      for (int b = 0; b < nb; b++) {
        const float x = tmem_ld1(lane_addr + (uint32_t)(c0 + b)) + __ldg(bias + c0 + b);
        cum += __expf(x - mx);
        if (!found && (cum > target || b == nb - 1)) {
          found = true;
          best = b;
          chosen = x;
        }
      }
    }
    logp += chosen - (mx + logf(se));
    if (valid) emit_choice(L, P.act_dim, row, g, best);
  }
  if (valid && L.logp) L.logp[row] = logp;
}

template <bool FP16>
__global__ void __launch_bounds__(THREADS, 1)
k_policy(const __grid_constant__ CUtensorMap xmap, const NetDev* __restrict__ nets_dev,
         const __grid_constant__ NetTable nets, const __grid_constant__ Launch L) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* act = base;
  uint8_t* stages = base + ACT_BYTES;
  Smem* S = reinterpret_cast<Smem*>(stages + STAGES * STAGE_BYTES);
  volatile int* abort_flag = &S->abort_flag;
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&S->x_full), 1);
    mbar_init(smem_u32(&S->act_empty), 1);
    mbar_init(smem_u32(&S->acc_full), 1);
    mbar_init(smem_u32(&S->acc_h0), 1);
    mbar_init(smem_u32(&S->act_ready), 32 * EPI_WARPS);
    mbar_init(smem_u32(&S->act_lo), 32 * EPI_WARPS);
    mbar_init(smem_u32(&S->tmem_empty), 32 * EPI_WARPS);
    mbar_init(smem_u32(&S->logp_bar), TILE_M * (EPI_PER_Q - 1));
    mbar_init(smem_u32(&S->drain), 1);
    for (int s = 0; s < STAGES; s++) {
      mbar_init(smem_u32(&S->full[s]), 1);
      mbar_init(smem_u32(&S->empty[s]), 1);
    }
    S->abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&S->tmem_base))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = S->tmem_base;
  const int64_t njobs = L.tiles_total * L.nets_per_group;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t it = 0;
      int64_t jn = 0;
      for (int64_t j = blockIdx.x; j < njobs; j += gridDim.x) {
        Job J;
        if (!decode_job(L, j, J)) continue;
        const NetParams& P = nets.p[J.net];
        const NetDev& D = nets_dev[J.net];
        // The input tile replaces the previous job's activations, so it waits until that job's
        // MMAs are done (act_empty); the weight ring does not: the first STAGES weight stages of
        // this job are requested before that wait, while the previous job's last layer runs.
        int sidx = 0;
        bool x_sent = false;
        auto send_x = [&]() -> bool {
          if (!mbar_wait(smem_u32(&S->act_empty), (uint32_t)((jn & 1) ^ 1), abort_flag)) return false;
          const int kc0 = P.in_pad / KCHUNK;
          mbar_expect_tx(smem_u32(&S->x_full), (uint32_t)(kc0 * TILE_M * 128));
          for (int c = 0; c < kc0; c++)
            tma_load_2d(smem_u32(act + c * TILE_M * 128), &xmap, c * KCHUNK, (int)J.row0, smem_u32(&S->x_full));
          x_sent = true;
          return true;
        };
        bool ok = true;
        for (int l = 0; l < P.n_layers - P.fold && ok; l++) {
          int K = (l == 0) ? P.in_pad : P.width_pad[l - 1];
          int N = P.width_pad[l];
          // every box of this layer's map moves box_rows x 128 B (rows past N arrive zero-filled);
          // cps boxes (consecutive K-chunks) share a stage
          const uint32_t box_bytes = (uint32_t)((N < NCHUNK ? N : NCHUNK) * 128);
          const int cps = chunks_per_stage(N, K);
          for (int n0 = 0; n0 < N && ok; n0 += NCHUNK) {
            for (int k0 = 0; k0 < K; k0 += cps * KCHUNK, it++) {
              int s = it % STAGES;
              uint32_t round = it / STAGES;
              const int nk = (K - k0) / KCHUNK < cps ? (K - k0) / KCHUNK : cps;
              if (!x_sent && sidx == STAGES && !send_x()) { ok = false; break; }
              sidx++;
              if (!mbar_wait(smem_u32(&S->empty[s]), (round & 1) ^ 1, abort_flag)) { ok = false; break; }
              mbar_expect_tx(smem_u32(&S->full[s]), box_bytes * (uint32_t)nk);
              for (int c = 0; c < nk; c++)
                tma_load_2d(smem_u32(stages + s * STAGE_BYTES + c * box_bytes), &D.w[l], k0 + c * KCHUNK, n0,
                            smem_u32(&S->full[s]));
            }
          }
        }
        if (ok && !x_sent && !send_x()) ok = false;
        if (!ok) break;
        jn++;
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      uint32_t it = 0, acts = 0, los = 0;
      bool prev_fold = false;
      int64_t jn = 0;
      for (int64_t j = blockIdx.x; j < njobs; j += gridDim.x) {
        Job J;
        if (!decode_job(L, j, J)) continue;
        const NetParams& P = nets.p[J.net];
        // Accumulator halves alternate between jobs: this job's first 256 output columns go to TMEM
        // columns side..side+255, the rest (and nothing of the previous job's head, which sat in
        // the other half) to the other half.  So the first layer's first half can be issued
        // while the previous job's output head is still being read, and only the first MMA
        // into the other half waits for that head (tmem_empty).
        const uint32_t side = (uint32_t)(jn & 1) << 8;
        bool tmem_ok = false;
        bool ok = mbar_wait(smem_u32(&S->x_full), (uint32_t)(jn & 1), abort_flag);
        // a folded value head kept both accumulator halves until its epilogue finished: no MMA of
        // this job before that epilogue has released them
        if (ok && prev_fold) {
          ok = mbar_wait(smem_u32(&S->tmem_empty), (uint32_t)((jn & 1) ^ 1), abort_flag);
          tmem_ok = true;
        }
        for (int l = 0; l < P.n_layers - P.fold && ok; l++) {
          int K = (l == 0) ? P.in_pad : P.width_pad[l - 1];
          int N = P.width_pad[l];
          const bool split = split_layer(P, l);
          const uint32_t box_bytes = (uint32_t)((N < NCHUNK ? N : NCHUNK) * 128);
          const int cps = chunks_per_stage(N, K);
          // After a split layer the epilogue releases its first 256 activations (and the TMEM
          // columns they came from) before the second half: this layer's K-chunks below K/2 can
          // start on act_lo, the rest wait for act_ready -- when K/2 falls on a stage boundary.
          const bool lo_first = l > 0 && split_layer(P, l - 1);
          const int k_hi = (lo_first && (K / 2) % (cps * KCHUNK) == 0) ? K / 2 : 0;
          if (lo_first) {
            if (!mbar_wait(smem_u32(&S->act_lo), los & 1, abort_flag)) { ok = false; break; }
            los++;
          }
          if (l > 0 && k_hi == 0) {
            if (!mbar_wait(smem_u32(&S->act_ready), acts & 1, abort_flag)) { ok = false; break; }
            acts++;
          }
          tc_fence_after();
          for (int n0 = 0; n0 < N && ok; n0 += NCHUNK) {
            int nc = (N - n0) < NCHUNK ? (N - n0) : NCHUNK;
            uint32_t idesc = idesc_f16<FP16>(nc);
            if (!tmem_ok && n0 >= NCHUNK) {
              if (!mbar_wait(smem_u32(&S->tmem_empty), (uint32_t)((jn & 1) ^ 1), abort_flag)) { ok = false; break; }
              tmem_ok = true;
            }
            for (int k0 = 0; k0 < K; k0 += cps * KCHUNK, it++) {
              int s = it % STAGES;
              uint32_t round = it / STAGES;
              const int nk = (K - k0) / KCHUNK < cps ? (K - k0) / KCHUNK : cps;
              if (n0 == 0 && k0 == k_hi && k_hi > 0) {
                if (!mbar_wait(smem_u32(&S->act_ready), acts & 1, abort_flag)) { ok = false; break; }
                acts++;
              }
              if (!mbar_wait(smem_u32(&S->full[s]), round & 1, abort_flag)) { ok = false; break; }
              tc_fence_after();
              for (int c = 0; c < nk; c++) {
                uint32_t a_base = smem_u32(act + (k0 / KCHUNK + c) * TILE_M * 128);
                uint32_t b_base = smem_u32(stages + s * STAGE_BYTES + c * box_bytes);
#pragma unroll
                for (int kk = 0; kk < KCHUNK / 16; kk++)
                  tc_mma(tmem + ((uint32_t)n0 ^ side), sdesc(a_base + kk * 32), sdesc(b_base + kk * 32), idesc,
                         (k0 > 0 || c > 0 || kk > 0) ? 1u : 0u);
              }
              tc_commit(smem_u32(&S->empty[s]));
            }
            if (split && n0 == 0) tc_commit(smem_u32(&S->acc_h0));
          }
          tc_commit(smem_u32(&S->acc_full));
        }
        // a job that never wrote the other half still consumes its tmem_empty phase
        if (ok && !tmem_ok && !mbar_wait(smem_u32(&S->tmem_empty), (uint32_t)((jn & 1) ^ 1), abort_flag)) ok = false;
        tc_commit(smem_u32(&S->act_empty));
        if (!ok) break;
        prev_fold = P.fold != 0;
        jn++;
      }
      // drain: wait (bounded) until every MMA this thread issued has completed
      tc_commit(smem_u32(&S->drain));
      long long t0 = clock64();
      while (!mbar_try(smem_u32(&S->drain), 0) && clock64() - t0 < WAIT_CYCLES) {
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2 and up)
    // Warp w may access TMEM lanes 32*(w%4)..+31 (its quarter of the tile rows); the EPI_PER_Q
    // warps of a quarter split the columns: part h takes the 32-column chunks with
    // index % EPI_PER_Q == h.
    const int q = warp & 3;
    const int h = (warp - 2) >> 2;
    const int m = q * 32 + lane;                  // tile row of this thread
    const uint32_t lane_addr = tmem + ((uint32_t)(q * 32) << 16);
    // the action grid, one entry per lane, for the categorical head's env commands
    const float grid_lane = (L.cmd && lane < 21) ? __ldg(L.grid + lane) : 0.0f;
    uint32_t accs = 0, heads = 0, h0s = 0;
    int64_t jn = 0;
    for (int64_t j = blockIdx.x; j < njobs; j += gridDim.x) {
      Job J;
      if (!decode_job(L, j, J)) continue;
      const NetParams& P = nets.p[J.net];
      bool ok = true;
      const uint32_t side = (uint32_t)(jn & 1) << 8;   // the MMA issuer's per-job accumulator half
      for (int l = 0; l < P.n_layers - P.fold; l++) {
        const bool split = split_layer(P, l);
        bool got = split ? mbar_wait(smem_u32(&S->acc_h0), h0s & 1, abort_flag)
                         : mbar_wait(smem_u32(&S->acc_full), accs & 1, abort_flag);
        __syncwarp();                               // reconverge before the .sync.aligned TMEM loads
        if (!got || *abort_flag) { ok = false; break; }
        if (split) h0s++;
        else accs++;
        tc_fence_after();
        const float* bias = P.bias[l];
        const bool last = (l == P.n_layers - 1);
        if (P.fold && l == P.n_layers - 2) {
          // the value head folded into the last hidden layer: each part dots its chunks' fp32
          // activations with the head's weights (the first half while the second half's MMAs
          // run), the quarter's parts join through shared memory, and both accumulator halves
          // are released together
          const int N = P.width_pad[l];
          const bool relu = P.act == 0;
          constexpr int STEP = 32 * EPI_PER_Q;
          // a split layer in two passes (the second after its last MMAs), one call site per
          // activation either way (compact code)
          float part = 0.0f;
          const int passes = split ? 2 : 1;
#pragma unroll 1
          for (int pass = 0; pass < passes; pass++) {
            if (pass == 1) {
              bool got2 = mbar_wait(smem_u32(&S->acc_full), accs & 1, abort_flag);
              __syncwarp();
              if (!got2 || *abort_flag) { ok = false; break; }
              accs++;
              tc_fence_after();
            }
            const int c0 = 32 * h + pass * NCHUNK, c1 = split ? (pass + 1) * NCHUNK : N;
            part = relu ? fold_chunks<FP16, true>(lane_addr, side, bias, P, c0, c1, STEP, part)
                        : fold_chunks<FP16, false>(lane_addr, side, bias, P, c0, c1, STEP, part);
          }
          if (!ok) break;
          const int64_t row = J.row0 + m;
          if (h != 0) {
            S->logp_part[h - 1][m] = part;
            mbar_arrive(smem_u32(&S->logp_bar));
          } else if (!mbar_wait(smem_u32(&S->logp_bar), heads & 1, abort_flag)) {
            ok = false;
          } else if (m < J.rows) {
#pragma unroll
            for (int k = 0; k < EPI_PER_Q - 1; k++) part += S->logp_part[k][m];
            const float val = part + __ldg(P.bias[P.n_layers - 1]);
            if (L.value) L.value[row] = val;
            if (L.logits) L.logits[row * L.logits_ld] = val;
          }
          heads++;
          tc_fence_before();
          mbar_arrive(smem_u32(&S->tmem_empty));
          if (!ok) break;
        } else if (!last) {
          // bias + activation -> bf16 into the swizzled A region of the next layer.  32-column
          // chunks, the TMEM load of the next chunk in flight while this one is converted.
          const int N = P.width_pad[l];
          const bool relu = P.act == 0;
          uint8_t* rowbase = act + (m >> 3) * 1024 + (m & 7) * 128;
          constexpr int STEP = 32 * EPI_PER_Q;           // this warp's chunks: c, c + STEP, ...
          int cstart = 32 * h;
          if (split) {
            // first half: packed to 16 bits and parked in the chunk's own (already read) TMEM
            // columns until the second half's MMAs are done with the activations being replaced
            constexpr int NH = NCHUNK / STEP;
#pragma unroll
            for (int i = 0; i < NH; i++) {
              const int c = cstart + i * STEP;
              ulonglong2 bv[8];
              load_bias32(bias, c, bv);
              uint32_t ra[32];
              tmem_ld32_nowait(lane_addr + ((uint32_t)c ^ side), ra);
              tmem_wait_ld();
              uint4 w[4];
              pack32<FP16>(ra, bv, relu, w);
              tmem_st16(lane_addr + ((uint32_t)c ^ side), w);
            }
            tmem_wait_st();
            bool got2 = mbar_wait(smem_u32(&S->acc_full), accs & 1, abort_flag);
            __syncwarp();
            if (!got2 || *abort_flag) { ok = false; break; }
            accs++;
            tc_fence_after();
#pragma unroll
            for (int i = 0; i < NH; i++) {
              const int c = cstart + i * STEP;
              uint4 w[4];
              tmem_ld16(lane_addr + ((uint32_t)c ^ side), w);
              store32(w, rowbase, c, m);
            }
            // the first half's activations are in place and its TMEM columns read: the next
            // layer's MMAs over them may start while the second half is converted
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            tc_fence_before();
            mbar_arrive(smem_u32(&S->act_lo));
            cstart += NCHUNK;
          }
          if (EPI_PER_Q >= 4) {
            // enough warps per scheduler to hide the TMEM load latency: one chunk at a time
            for (int c = cstart; c < N; c += STEP) {
              ulonglong2 bv[8];
              load_bias32(bias, c, bv);
              uint32_t ra[32];
              tmem_ld32_nowait(lane_addr + ((uint32_t)c ^ side), ra);
              tmem_wait_ld();
              convert32<FP16>(ra, bv, c, rowbase, m, relu);
            }
          } else {
            // the next chunk's TMEM load in flight while this one is converted
            uint32_t ra[32], rb[32];
            int c = cstart;
            if (c < N) {
              tmem_ld32_nowait(lane_addr + ((uint32_t)c ^ side), ra);
              tmem_wait_ld();
            }
            while (c < N) {
              if (c + STEP < N) tmem_ld32_nowait(lane_addr + ((uint32_t)(c + STEP) ^ side), rb);
              { ulonglong2 bv[8]; load_bias32(bias, c, bv); convert32<FP16>(ra, bv, c, rowbase, m, relu); }
              tmem_wait_ld();
              c += STEP;
              if (c >= N) break;
              if (c + STEP < N) tmem_ld32_nowait(lane_addr + ((uint32_t)(c + STEP) ^ side), ra);
              { ulonglong2 bv[8]; load_bias32(bias, c, bv); convert32<FP16>(rb, bv, c, rowbase, m, relu); }
              tmem_wait_ld();
              c += STEP;
            }
          }
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          tc_fence_before();
          mbar_arrive(smem_u32(&S->act_ready));
        } else {
          const int64_t row = J.row0 + m;
          const bool valid = m < J.rows;
          if (P.head == HEAD_VALUE) {
            if (h == 0) {
              float v[32];
              tmem_ld32(lane_addr + side, v);
              float val = v[0] + __ldg(bias);
              if (valid) {
                if (L.value) L.value[row] = val;
                if (L.logits) L.logits[row * L.logits_ld] = val;
              }
            }
          } else if (P.act_dim == 4 && P.num_bins == 21) {
            // the channels split over the quarter's parts; the other parts' log-probs join part 0
            // through shared memory
            if (h != 0) {
              float part;
              if (EPI_PER_Q == 4) part = cat_head1<4, 21>(lane_addr + side, bias, L, row, valid, grid_lane, h);
              else part = cat_head<4, 21, 1, EPI_PER_Q>(lane_addr + side, bias, L, row, valid, grid_lane);
              S->logp_part[h - 1][m] = part;
              mbar_arrive(smem_u32(&S->logp_bar));
            } else {
              float part = EPI_PER_Q == 4 ? cat_head1<4, 21>(lane_addr + side, bias, L, row, valid, grid_lane, 0)
                                          : cat_head<4, 21, 0, EPI_PER_Q>(lane_addr + side, bias, L, row, valid, grid_lane);
              if (!mbar_wait(smem_u32(&S->logp_bar), heads & 1, abort_flag)) {
                ok = false;
              } else if (valid && L.logp) {
#pragma unroll
                for (int k = 0; k < EPI_PER_Q - 1; k++) part += S->logp_part[k][m];
                L.logp[row] = part;
              }
            }
            heads++;
          } else if (h == 0) {
            cat_head_generic(lane_addr + side, bias, L, P, row, valid);
          }
          tc_fence_before();
          mbar_arrive(smem_u32(&S->tmem_empty));
          if (!ok) break;
        }
      }
      if (!ok) break;
      jn++;
    }
  }

  // ---------------------------------------------------------------- teardown
  __syncwarp();
  if (*abort_flag) {
    // a role gave up waiting: give copies still in flight a bounded time to land before exit
    for (int i = 0; i < 4; i++) __nanosleep(1000000);
  }
  tc_fence_before();
  __syncthreads();
  if (*abort_flag && threadIdx.x == 0 && L.err) atomicExch(L.err, F16_ERR_LAUNCH);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(tmem) : "memory");
  }
}

// ---------------------------------------------------------------- host side
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// 16-bit (bf16 or fp16) row-major [rows][cols] (row stride ld elements) with a 128-byte-swizzled
// box of 64 x box_rows
static bool make_map(CUtensorMap* m, const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows,
                     bool fp16) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)KCHUNK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(m, fp16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace mlp
}  // namespace f16

struct f16_mlp_set_s {
  int n;
  int fp16;                        // operand type of every network in the set
  f16::mlp::NetDev* dev_maps;      // device [n]
  // host copy of every network's parameters, passed to each launch by value
  f16::mlp::NetParams host_params[f16::mlp::MAX_NETS];
};

using namespace f16;
using namespace f16::mlp;

extern "C" int f16_mlp_set_create(const f16_mlp_desc* descs, int n, f16_mlp_set** out) {
  if (!descs || n <= 0 || n > MAX_NETS || !out) return F16_ERR_ARG;
  *out = nullptr;
  NetDev maps[MAX_NETS];
  f16_mlp_set_s* s = new f16_mlp_set_s();
  s->n = n;
  for (int i = 0; i < n; i++) {
    const f16_mlp_desc& d = descs[i];
    NetParams& P = s->host_params[i];
    memset(&P, 0, sizeof(P));
    if (d.n_layers < 1 || d.n_layers > MAX_LAYERS || d.in_dim <= 0 || d.in_dim % 8 != 0 || d.in_dim > 512 ||
        (d.activation != 0 && d.activation != 1) || (d.head != HEAD_CATEGORICAL && d.head != HEAD_VALUE) ||
        (d.operand != F16_OPERAND_BF16 && d.operand != F16_OPERAND_FP16) || d.operand != descs[0].operand) {
      delete s;
      return F16_ERR_ARG;
    }
    P.fp16 = d.operand == F16_OPERAND_FP16;
    s->fp16 = P.fp16;
    P.n_layers = d.n_layers;
    P.in_pad = (d.in_dim + KCHUNK - 1) / KCHUNK * KCHUNK;
    P.act = d.activation;
    P.head = d.head;
    P.num_bins = d.num_bins;
    P.act_dim = d.act_dim;
    int in_l = d.in_dim;
    for (int l = 0; l < d.n_layers; l++) {
      int w = d.width[l];
      bool last = (l == d.n_layers - 1);
      if (!d.weight[l] || !d.bias[l] || w <= 0) { delete s; return F16_ERR_ARG; }
      if (!aligned(d.weight[l], 16)) { delete s; return F16_ERR_ALIGN; }
      if (!last && (w % KCHUNK != 0 || w > 512)) { delete s; return F16_ERR_ARG; }
      int wp = last ? (w + 15) / 16 * 16 : w;
      if (last && d.head == HEAD_CATEGORICAL && (wp > 96 || d.act_dim * d.num_bins != w || d.num_bins > 64)) {
        delete s;
        return F16_ERR_ARG;
      }
      if (last && d.head == HEAD_VALUE && w != 1) { delete s; return F16_ERR_ARG; }
      P.width[l] = w;
      P.width_pad[l] = wp;
      P.bias[l] = d.bias[l];
      int box_rows = wp < NCHUNK ? wp : NCHUNK;
      if (!make_map(&maps[i].w[l], d.weight[l], w, in_l, in_l, box_rows, P.fp16 != 0)) {
        delete s;
        return F16_ERR_CUDA;
      }
      in_l = w;
    }
    P.fold = (d.head == HEAD_VALUE && d.n_layers >= 2) ? 1 : 0;
    P.head_w16 = d.weight[d.n_layers - 1];
    P.head_w32 = d.head_weight_f32;
    if (P.head_w32 && !aligned(P.head_w32, 16)) { delete s; return F16_ERR_ALIGN; }
  }
  if (cudaMalloc(&s->dev_maps, sizeof(NetDev) * n) != cudaSuccess) {
    delete s;
    return F16_ERR_CUDA;
  }
  if (cudaMemcpy(s->dev_maps, maps, sizeof(NetDev) * n, cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(s->dev_maps);
    delete s;
    return F16_ERR_CUDA;
  }
  *out = s;
  return F16_OK;
}

extern "C" int f16_mlp_set_destroy(f16_mlp_set* s) {
  if (!s) return F16_ERR_ARG;
  cudaFree(s->dev_maps);
  delete s;
  return F16_OK;
}

extern "C" int f16_policy_forward(const f16_mlp_set* set, const f16_policy_args* a, f16_stream_t stream) {
  if (!set || !a || !a->x || a->rows <= 0 || a->n_groups < 1 || a->n_groups > MAX_NETS || !a->group_end ||
      !a->group_net || a->nets_per_group < 1 || a->nets_per_group > 2)
    return F16_ERR_ARG;
  if (!aligned(a->x, 16) || (a->ldx * 2) % 16 != 0) return F16_ERR_ALIGN;
  Launch L;
  memset(&L, 0, sizeof(L));
  L.rows = a->rows;
  L.n_groups = a->n_groups;
  L.nets_per_group = a->nets_per_group;
  int64_t start = 0, tiles = 0;
  int in_pad = -1;
  const bool dev_ends = a->group_end_dev != nullptr;
  if (dev_ends && !aligned(a->group_end_dev, 8)) return F16_ERR_ALIGN;
  L.group_end_dev = a->group_end_dev;
  for (int g = 0; g < a->n_groups; g++) {
    if (!dev_ends) {
      int64_t end = a->group_end[g];
      if (end < start || end > a->rows || start % TILE_M != 0) return F16_ERR_ARG;
      L.group_end[g] = end;
      tiles += (end - start + TILE_M - 1) / TILE_M;
      start = end;
    }
    for (int k = 0; k < 2; k++) {
      int net = k < a->nets_per_group ? a->group_net[g * a->nets_per_group + k] : -1;
      if (net >= set->n) return F16_ERR_ARG;
      if (net >= 0) {
        int ip = set->host_params[net].in_pad;
        if (in_pad >= 0 && ip != in_pad) return F16_ERR_ARG;
        in_pad = ip;
        if (set->host_params[net].head == HEAD_CATEGORICAL && (!a->logp && !a->bins && !a->act_idx && !a->logits && !a->cmd))
          return F16_ERR_ARG;
      }
      L.group_net[g][k] = net;
    }
  }
  // device-resident ends: every tile of every group lies in [0, rows), at most one partial tile
  // per group
  if (dev_ends) tiles = (a->rows + TILE_M - 1) / TILE_M + a->n_groups;
  if (in_pad < 0 || a->ldx < 8) return F16_ERR_ARG;
  L.tiles_total = tiles;
  L.bins = a->bins; L.bins_stride = a->bins_stride; L.bins_offset = a->bins_offset;
  L.act_idx = a->act_idx; L.logp = a->logp; L.value = a->value;
  L.logits = a->logits; L.logits_ld = a->logits_ld;
  L.seed = a->seed; L.step = a->step; L.step_dev = a->step_dev; L.deterministic = a->deterministic;
  L.err = a->err;
  if (a->cmd && (!a->grid || a->cmd_stride < 0 || a->cmd_offset < 0)) return F16_ERR_ARG;
  L.cmd = a->cmd; L.cmd_stride = a->cmd_stride; L.cmd_offset = a->cmd_offset; L.grid = a->grid;
  CUtensorMap xmap;
  if (!make_map(&xmap, a->x, a->rows, a->ldx, a->ldx, TILE_M, set->fp16 != 0)) return F16_ERR_CUDA;
  int64_t njobs = tiles * a->nets_per_group;
  if (njobs == 0) return F16_OK;
  static bool attr[2][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  const int t = set->fp16 ? 1 : 0;
  if (dev >= 0 && dev < 64 && !attr[t][dev]) {
    cudaError_t e = t ? cudaFuncSetAttribute(k_policy<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES)
                      : cudaFuncSetAttribute(k_policy<false>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return F16_ERR_LAUNCH;
    attr[t][dev] = true;
  }
  int grid = (int)(njobs < sm_count() ? njobs : sm_count());
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  NetTable nets;
  memset(&nets, 0, sizeof(nets));
  memcpy(nets.p, set->host_params, sizeof(NetParams) * set->n);
  if (t) k_policy<true><<<grid, THREADS, SMEM_BYTES, st>>>(xmap, set->dev_maps, nets, L);
  else k_policy<false><<<grid, THREADS, SMEM_BYTES, st>>>(xmap, set->dev_maps, nets, L);
  return launch_status();
}
