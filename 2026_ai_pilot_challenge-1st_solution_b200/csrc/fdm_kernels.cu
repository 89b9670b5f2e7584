// fdm_kernels.cu -- FDM+FCS step and GPU IC seeder kernels, with their C-ABI entry points.
//
// Kernel shape (B200, sm_100a): one thread per aircraft, persistent grid of
// (SM count x resident blocks) iterating over aircraft with a grid stride.  State is read once
// per launch (coalesced when SoA), kept in registers across the `substeps` frames, and written
// once; of the four 3-deep integrator histories only the slots that survive the launch are
// stored.  The 11.9 KB coefficient image is staged per block in shared memory.
#include "common.cuh"
#include "fdm_device.cuh"

namespace f16 {

// Launch shape: 256 threads x 2 resident blocks per SM caps the kernel at 128 registers
// (16 warps/SM).  Measured on B200 for the cfg2 step (131,072 aircraft, 6 frames):
// 128x3 (168 regs) 0.304 ms, 128x4 0.259 ms, 128x5 (96 regs) 0.286 ms, 256x2 0.253 ms; at higher
// occupancy the spills win nothing back: 256x3 (85 regs) 1.9e9 frames/s, 256x4 / 128x8
// (64 regs) 2.3e9 / 2.2e9 against 3.0e9 for 256x2.
#ifndef F16_FDM_MIN_BLOCKS
#define F16_FDM_MIN_BLOCKS 2
#endif
constexpr int FDM_MIN_BLOCKS = F16_FDM_MIN_BLOCKS;
constexpr size_t FDM_SMEM = SMEM_DOUBLES * sizeof(double);

// Per-bin command values of the reference action grid (R/cuda_fdm/ppo_gpu.py:178-180, 361-369):
// channel value = float32 linspace(-1, 1, nb)[i], throttle = 0.5*v + 0.5 in float32.
struct BinGrid {
  double ch[64];
  double thr[64];
};

template <int LAYOUT>
__device__ __forceinline__ void load_state(const StateRef<LAYOUT>& R, int64_t a, Ac& s) {
#pragma unroll
  for (int i = 0; i < 3; i++) {
    s.pos[i] = R(a, F16_S_POS + i);
    s.vel[i] = R(a, F16_S_VEL + i);
    s.pqri[i] = R(a, F16_S_PQRI + i);
    s.uvwidot[i] = R(a, F16_S_UVWIDOT + i);
    s.pqridot[i] = R(a, F16_S_PQRIDOT + i);
    s.ivel1[i] = R(a, F16_S_DEQ_IVEL + i);
    s.ivel2[i] = R(a, F16_S_DEQ_IVEL + 3 + i);
    s.uvd1[i] = R(a, F16_S_DEQ_UVWIDOT + i);
    s.pbacc[i] = R(a, F16_S_PREV_BACC + i);
    s.ppqridot[i] = R(a, F16_S_PREV_PQRIDOT + i);
    s.ppqri[i] = R(a, F16_S_PREV_PQRI + i);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    s.q[i] = R(a, F16_S_Q + i);
    s.qdot[i] = R(a, F16_S_QDOT + i);
    s.eng[i] = R(a, F16_S_ENG + i);
  }
  s.epa = R(a, F16_S_EPA);
  s.fuel = R(a, F16_S_FUEL);
#pragma unroll
  for (int i = 0; i < 9; i++) {
    s.pa[i] = R(a, F16_S_PREV_AUX + i);
    s.pid[i] = R(a, F16_S_PID + i);
  }
#pragma unroll
  for (int i = 0; i < 6; i++) s.kin[i] = R(a, F16_S_KIN + i);
  load_factor(s.fuel, s.pbacc, s.ppqridot, s.ppqri, s.nld);
}

// Non-finite test on the exponent bits (all-ones exponent = inf or NaN); `bad` ORs it up.  The
// kernels that report no finite flag are built with CHECK = false and skip the test.
template <bool CHECK = true>
__device__ __forceinline__ double fin(double v, unsigned& bad) {
  if (CHECK) bad |= (unsigned)((__double2hiint(v) & 0x7ff00000) == 0x7ff00000);
  return v;
}

template <int LAYOUT, bool CHECK = true>
__device__ __forceinline__ void store_state(const StateRef<LAYOUT>& R, int64_t a, const Ac& s, unsigned& bad) {
#pragma unroll
  for (int i = 0; i < 3; i++) {
    R(a, F16_S_POS + i) = fin<CHECK>(s.pos[i], bad);
    R(a, F16_S_VEL + i) = fin<CHECK>(s.vel[i], bad);
    R(a, F16_S_PQRI + i) = fin<CHECK>(s.pqri[i], bad);
    R(a, F16_S_UVWIDOT + i) = fin<CHECK>(s.uvwidot[i], bad);
    R(a, F16_S_PQRIDOT + i) = fin<CHECK>(s.pqridot[i], bad);
    R(a, F16_S_PREV_BACC + i) = fin<CHECK>(s.pbacc[i], bad);
    R(a, F16_S_PREV_PQRIDOT + i) = fin<CHECK>(s.ppqridot[i], bad);
    R(a, F16_S_PREV_PQRI + i) = fin<CHECK>(s.ppqri[i], bad);
  }
#pragma unroll
  for (int i = 0; i < 4; i++) {
    R(a, F16_S_Q + i) = fin<CHECK>(s.q[i], bad);
    R(a, F16_S_QDOT + i) = fin<CHECK>(s.qdot[i], bad);
    R(a, F16_S_ENG + i) = fin<CHECK>(s.eng[i], bad);
  }
  R(a, F16_S_EPA) = fin<CHECK>(s.epa, bad);
  R(a, F16_S_FUEL) = fin<CHECK>(s.fuel, bad);
#pragma unroll
  for (int i = 0; i < 9; i++) {
    R(a, F16_S_PREV_AUX + i) = fin<CHECK>(s.pa[i], bad);
    R(a, F16_S_PID + i) = fin<CHECK>(s.pid[i], bad);
  }
#pragma unroll
  for (int i = 0; i < 6; i++) R(a, F16_S_KIN + i) = fin<CHECK>(s.kin[i], bad);
}

template <int LAYOUT>
__device__ __forceinline__ void store_state(const StateRef<LAYOUT>& R, int64_t a, const Ac& s) {
  unsigned bad = 0;
  store_state(R, a, s, bad);
}

// Store the values pushed into the four integrator histories in frame i into the deque slot
// j = substeps-1-i they occupy when the launch ends (only slots j <= 2 exist).
template <int LAYOUT, bool CHECK = true>
__device__ __forceinline__ void store_history(const StateRef<LAYOUT>& R, int64_t a, int j, const Ac& s,
                                              unsigned& bad) {
#pragma unroll
  for (int i = 0; i < 4; i++) R(a, F16_S_DEQ_Q + 4 * j + i) = fin<CHECK>(s.qdot[i], bad);
#pragma unroll
  for (int i = 0; i < 3; i++) {
    R(a, F16_S_DEQ_PQRI + 3 * j + i) = fin<CHECK>(s.pqridot[i], bad);
    R(a, F16_S_DEQ_IVEL + 3 * j + i) = fin<CHECK>(s.vel[i], bad);
    R(a, F16_S_DEQ_UVWIDOT + 3 * j + i) = fin<CHECK>(s.uvwidot[i], bad);
  }
}

template <int LAYOUT>
__device__ __forceinline__ void store_history(const StateRef<LAYOUT>& R, int64_t a, int j, const Ac& s) {
  unsigned bad = 0;
  store_history(R, a, j, s, bad);
}

// With fewer than 3 frames per launch the oldest surviving slots are the old ones shifted.
template <int LAYOUT, bool CHECK = true>
__device__ __forceinline__ void shift_old_history(const StateRef<LAYOUT>& R, int64_t a, int substeps, unsigned& bad) {
  if (substeps >= 3) return;
  double q0[4], q1[4], p0[3], p1[3], v0[3], v1[3], u0[3], u1[3];
#pragma unroll
  for (int i = 0; i < 4; i++) { q0[i] = R(a, F16_S_DEQ_Q + i); q1[i] = R(a, F16_S_DEQ_Q + 4 + i); }
#pragma unroll
  for (int i = 0; i < 3; i++) {
    p0[i] = R(a, F16_S_DEQ_PQRI + i); p1[i] = R(a, F16_S_DEQ_PQRI + 3 + i);
    v0[i] = R(a, F16_S_DEQ_IVEL + i); v1[i] = R(a, F16_S_DEQ_IVEL + 3 + i);
    u0[i] = R(a, F16_S_DEQ_UVWIDOT + i); u1[i] = R(a, F16_S_DEQ_UVWIDOT + 3 + i);
  }
  // slot j <- old slot j - substeps, for j = substeps..2
  for (int j = substeps; j <= 2; j++) {
    int o = j - substeps;
#pragma unroll
    for (int i = 0; i < 4; i++) R(a, F16_S_DEQ_Q + 4 * j + i) = fin<CHECK>(o == 0 ? q0[i] : q1[i], bad);
#pragma unroll
    for (int i = 0; i < 3; i++) {
      R(a, F16_S_DEQ_PQRI + 3 * j + i) = fin<CHECK>(o == 0 ? p0[i] : p1[i], bad);
      R(a, F16_S_DEQ_IVEL + 3 * j + i) = fin<CHECK>(o == 0 ? v0[i] : v1[i], bad);
      R(a, F16_S_DEQ_UVWIDOT + 3 * j + i) = fin<CHECK>(o == 0 ? u0[i] : u1[i], bad);
    }
  }
}

template <int LAYOUT, bool BINS, bool CHECK>
__global__ void __launch_bounds__(FDM_THREADS, FDM_MIN_BLOCKS)
k_fdm_step(double* __restrict__ st, int64_t ld, int64_t nac, const double* __restrict__ cmd,
           const uint8_t* __restrict__ bins, const BinGrid grid, int substeps, double fcs_dt,
           double* __restrict__ obs17, uint8_t* __restrict__ finite) {
  extern __shared__ double S[];
  stage_tables(S);
  const double inv_fcs_dt = 1.0 / fcs_dt;
  const double gear = gear_actuator(fcs_dt);
  StateRef<LAYOUT> R{st, ld};
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; a < nac; a += stride) {
    double c0, c1, c2, c3;
    if (BINS) {
      uchar4 b = reinterpret_cast<const uchar4*>(bins)[a];
      c0 = grid.ch[b.x]; c1 = grid.ch[b.y]; c2 = grid.ch[b.z]; c3 = grid.thr[b.w];
    } else {
      const double2* cp = reinterpret_cast<const double2*>(cmd + 4 * a);
      double2 x = cp[0], y = cp[1];
      c0 = x.x; c1 = x.y; c2 = y.x; c3 = y.y;
    }
    Ac s;
    unsigned bad = 0;                       // any stored state value non-finite
    load_state(R, a, s);
    shift_old_history<LAYOUT, CHECK>(R, a, substeps, bad);
    FrameOut out;
    for (int i = 0; i < substeps - 1; i++) {
      int j = substeps - 1 - i;
      if (j <= 2) store_history<LAYOUT, CHECK>(R, a, j, s, bad);
      propagate(s);
      dynamics(S, s, c0, c1, c2, c3, fcs_dt, inv_fcs_dt, gear, out, false);
    }
    store_history<LAYOUT, CHECK>(R, a, 0, s, bad);
    propagate(s);
    dynamics(S, s, c0, c1, c2, c3, fcs_dt, inv_fcs_dt, gear, out, true);
    store_state<LAYOUT, CHECK>(R, a, s, bad);
    if (CHECK) finite[a] = bad ? 0 : 1;
    if (obs17) {
      double* o = obs17 + 17 * a;
      o[0] = s.pos[0]; o[1] = s.pos[1]; o[2] = s.pos[2];
      o[3] = s.vel[0]; o[4] = s.vel[1]; o[5] = s.vel[2];
      o[6] = out.euler[0]; o[7] = out.euler[1]; o[8] = out.euler[2];
      o[9] = out.uvw[0]; o[10] = out.uvw[1]; o[11] = out.uvw[2];
      o[12] = out.alpha; o[13] = out.beta; o[14] = out.mach; o[15] = out.vt; o[16] = out.alt;
    }
  }
}

// ---------------- IC seeder (cuda_fdm/ic.py:18-138, cuda_fdm/ref/jsb_fdm.py:142-210) ----------------
__device__ __forceinline__ void mat3_mul(const double A[3][3], const double B[3][3], double O[3][3]) {
  for (int i = 0; i < 3; i++)
    for (int j = 0; j < 3; j++) O[i][j] = A[i][0] * B[0][j] + A[i][1] * B[1][j] + A[i][2] * B[2][j];
}
__device__ void q_to_dcm(const double q[4], double M[3][3]) {
  double a = q[0], b = q[1], c = q[2], d = q[3];
  double aa = a * a, bb = b * b, cc = c * c, dd = d * d;
  double ab = a * b, ac = a * c, ad = a * d, bc = b * c, bd = b * d, cd = c * d;
  M[0][0] = aa + bb - cc - dd; M[0][1] = 2.0 * (bc + ad); M[0][2] = 2.0 * (bd - ac);
  M[1][0] = 2.0 * (bc - ad); M[1][1] = aa - bb + cc - dd; M[1][2] = 2.0 * (cd + ab);
  M[2][0] = 2.0 * (bd + ac); M[2][1] = 2.0 * (cd - ab); M[2][2] = aa - bb - cc + dd;
}
__device__ void dcm_to_q(const double m[3][3], double Q[4]) {
  // JSBSim FGMatrix33::GetQuaternion on the column-major element order (fdm.cuh:113-121)
  double c[9] = {m[0][0], m[1][0], m[2][0], m[0][1], m[1][1], m[2][1], m[0][2], m[1][2], m[2][2]};
  double t[4] = {1.0 + c[0] + c[4] + c[8], 1.0 + c[0] - c[4] - c[8], 1.0 - c[0] + c[4] - c[8],
                 1.0 - c[0] - c[4] + c[8]};
  int k = 0;
  for (int i = 1; i < 4; i++)
    if (t[i] > t[k]) k = i;
  if (k == 0) {
    Q[0] = 0.5 * sqrt(t[0]);
    Q[1] = 0.25 * (c[7] - c[5]) / Q[0]; Q[2] = 0.25 * (c[2] - c[6]) / Q[0]; Q[3] = 0.25 * (c[3] - c[1]) / Q[0];
  } else if (k == 1) {
    Q[1] = 0.5 * sqrt(t[1]);
    Q[0] = 0.25 * (c[7] - c[5]) / Q[1]; Q[2] = 0.25 * (c[3] + c[1]) / Q[1]; Q[3] = 0.25 * (c[2] + c[6]) / Q[1];
  } else if (k == 2) {
    Q[2] = 0.5 * sqrt(t[2]);
    Q[0] = 0.25 * (c[2] - c[6]) / Q[2]; Q[1] = 0.25 * (c[3] + c[1]) / Q[2]; Q[3] = 0.25 * (c[7] + c[5]) / Q[2];
  } else {
    Q[3] = 0.5 * sqrt(t[3]);
    Q[0] = 0.25 * (c[3] - c[1]) / Q[3]; Q[1] = 0.25 * (c[6] + c[2]) / Q[3]; Q[2] = 0.25 * (c[7] + c[5]) / Q[3];
  }
}

template <int LAYOUT>
__global__ void __launch_bounds__(FDM_THREADS, FDM_MIN_BLOCKS)
k_seed_ic(const double* __restrict__ ic, int64_t nac, double* __restrict__ st, int64_t ld, double fcs_dt) {
  extern __shared__ double S[];
  stage_tables(S);
  const double gear = gear_actuator(fcs_dt);
  StateRef<LAYOUT> R{st, ld};
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t a = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; a < nac; a += stride) {
    const double* in = ic + F16_IC_N * a;
    const double d2r = M_PI / 180.0;
    double lat = in[F16_IC_LAT_DEG] * d2r, lon = in[F16_IC_LON_DEG] * d2r, alt = in[F16_IC_ALT_FT];
    double vt = in[F16_IC_VT_FPS];
    double phi = in[F16_IC_PHI_DEG] * d2r, tht = in[F16_IC_THETA_DEG] * d2r, psi = in[F16_IC_PSI_DEG] * d2r;
    double al = in[F16_IC_ALPHA_DEG] * d2r, be = in[F16_IC_BETA_DEG] * d2r;
    double fuel = in[F16_IC_FUEL_LBS], ff = in[F16_IC_FUELFLOW_PPH];
    double e[3];
    double slat = sin(lat), clat = cos(lat), slon = sin(lon), clon = cos(lon);
    if (in[F16_IC_GEOCENTRIC] != 0.0) {
      double rr = F16C_SEMI_MAJOR + alt;
      e[0] = rr * clat * clon; e[1] = rr * clat * slon; e[2] = rr * slat;
    } else {
      // point on the WGS84 normal through (lat,lon) with |ecef| = a + alt (ic.py:18-39)
      double A0 = F16C_SEMI_MAJOR, e2 = F16C_E2;
      double N = A0 / sqrt(1.0 - e2 * slat * slat);
      double A = clat * clat, B = slat * slat, P = N, Qv = N * (1.0 - e2);
      double b = A * P + B * Qv, c = A * P * P + B * Qv * Qv, Rr = A0 + alt;
      double t = -b + sqrt(b * b - c + Rr * Rr);
      e[0] = (N + t) * clat * clon; e[1] = (N + t) * clat * slon; e[2] = (N * (1.0 - e2) + t) * slat;
    }
    // epa = 0: ECI coincides with ECEF.  Local frame from the position (fdm.cuh:140-153).
    double x = e[0], y = e[1], z = e[2];
    double r = sqrt(x * x + y * y + z * z), rxy = sqrt(x * x + y * y);
    double sLo, cLo, sLa, cLa;
    if (rxy == 0.0) { sLo = 0.0; cLo = 1.0; } else { sLo = y / rxy; cLo = x / rxy; }
    if (r == 0.0) { sLa = 0.0; cLa = 1.0; } else { sLa = z / r; cLa = rxy / r; }
    double Ti2l[3][3] = {{-cLo * sLa, -sLo * sLa, cLa}, {-sLo, cLo, 0.0}, {-cLo * cLa, -sLo * cLa, -sLa}};
    double qL[4], Tl2b[3][3], Ti2b[3][3];
    {
      double st_ = sin(0.5 * tht), sp = sin(0.5 * psi), sf = sin(0.5 * phi);
      double ct = cos(0.5 * tht), cp = cos(0.5 * psi), cf = cos(0.5 * phi);
      double cfct = cf * ct, cfst = cf * st_, sfst = sf * st_, sfct = sf * ct;
      qL[0] = cfct * cp + sfst * sp; qL[1] = sfct * cp - cfst * sp;
      qL[2] = cfst * cp + sfct * sp; qL[3] = cfct * sp - sfst * cp;
      double m = sqrt(qL[0] * qL[0] + qL[1] * qL[1] + qL[2] * qL[2] + qL[3] * qL[3]);
      if (m != 0.0) { double k = 1.0 / m; qL[0] *= k; qL[1] *= k; qL[2] *= k; qL[3] *= k; }
    }
    q_to_dcm(qL, Tl2b);
    mat3_mul(Tl2b, Ti2l, Ti2b);
    Ac s;
    double uvw[3] = {vt * cos(al) * cos(be), vt * sin(be), vt * sin(al) * cos(be)};
    for (int i = 0; i < 3; i++) {
      s.pos[i] = e[i];
      s.vel[i] = Ti2b[0][i] * uvw[0] + Ti2b[1][i] * uvw[1] + Ti2b[2][i] * uvw[2];
    }
    s.vel[0] += -ROT * y;
    s.vel[1] += ROT * x;
    dcm_to_q(Ti2b, s.q);
    for (int i = 0; i < 3; i++) s.pqri[i] = 0.0 + Ti2b[i][2] * ROT;
    s.epa = 0.0;
    s.fuel = fuel;
    // prev_aux from the IC (ic.py:127-132)
    Air at;
    isa(S, alt, at);
    double mach = vt * at.ia;
    s.pa[0] = al; s.pa[1] = mach; s.pa[2] = vcas_kts(mach, at.P); s.pa[3] = vt; s.pa[4] = 0.0;
    s.pa[5] = -1.0; s.pa[6] = 0.0; s.pa[7] = 0.0; s.pa[8] = 0.0;
    double pa_ic[9];
    for (int i = 0; i < 9; i++) pa_ic[i] = s.pa[i];
    // throwaway force path: fresh FCS, fresh engine with the IC fuel flow, commands (0,0,0,0.8)
    for (int i = 0; i < 6; i++) s.kin[i] = 0.0;
    for (int i = 0; i < 9; i++) s.pid[i] = 0.0;
    s.eng[0] = 100.0; s.eng[1] = 100.0; s.eng[2] = (100.0 - F16C_IDLEN2) / (F16C_MAXN2 - F16C_IDLEN2); s.eng[3] = ff;
    for (int i = 0; i < 3; i++) { s.pbacc[i] = 0.0; s.ppqridot[i] = 0.0; s.ppqri[i] = s.pqri[i]; }
    load_factor(s.fuel, s.pbacc, s.ppqridot, s.ppqri, s.nld);
    FrameOut out;
    dynamics(S, s, 0.0, 0.0, 0.0, 0.8, fcs_dt, 1.0 / fcs_dt, gear, out, true);
    // outputs: the derivatives; everything else returns to the fresh / IC values
    s.fuel = fuel;
    for (int i = 0; i < 9; i++) s.pa[i] = pa_ic[i];
    for (int i = 0; i < 6; i++) s.kin[i] = 0.0;
    for (int i = 0; i < 9; i++) s.pid[i] = 0.0;
    s.eng[0] = 100.0; s.eng[1] = 100.0; s.eng[2] = (100.0 - F16C_IDLEN2) / (F16C_MAXN2 - F16C_IDLEN2); s.eng[3] = ff;
    for (int i = 0; i < 3; i++) { s.ivel1[i] = s.vel[i]; s.ivel2[i] = s.vel[i]; s.uvd1[i] = s.uvwidot[i]; }
    store_state(R, a, s);
    for (int j = 0; j < 3; j++) store_history(R, a, j, s);
  }
}

// ---------------- launch helpers ----------------
template <typename K>
int persistent_grid(K kernel, int64_t nac, size_t smem) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, FDM_THREADS, smem) != cudaSuccess || per_sm < 1)
    per_sm = 1;
  int64_t need = (nac + FDM_THREADS - 1) / FDM_THREADS;
  int64_t cap = (int64_t)sm_count() * per_sm;
  return (int)(need < cap ? need : cap);
}

template <int LAYOUT, bool BINS>
int launch_step(double* st, int64_t ld, int64_t nac, const double* cmd, const uint8_t* bins, const BinGrid& g,
                int substeps, double fcs_dt, double* obs17, cudaStream_t stream, uint8_t* finite = nullptr) {
  auto k = finite ? k_fdm_step<LAYOUT, BINS, true> : k_fdm_step<LAYOUT, BINS, false>;
  static bool attr_set[2][64] = {{false}};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !attr_set[finite ? 1 : 0][dev]) {
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FDM_SMEM);
    attr_set[finite ? 1 : 0][dev] = true;
  }
  int grid = persistent_grid(k, nac, FDM_SMEM);
  k<<<grid, FDM_THREADS, FDM_SMEM, stream>>>(st, ld, nac, cmd, bins, g, substeps, fcs_dt, obs17, finite);
  return launch_status();
}

int check_state_args(const double* state, int layout, int64_t ld, int64_t nac) {
  if (!state || nac <= 0) return F16_ERR_ARG;
  if (layout != F16_LAYOUT_SOA && layout != F16_LAYOUT_AOS) return F16_ERR_ARG;
  if (layout == F16_LAYOUT_SOA && ld < nac) return F16_ERR_ARG;
  if (!aligned(state, 8)) return F16_ERR_ALIGN;
  return F16_OK;
}

}  // namespace f16

using namespace f16;

extern "C" int f16_fdm_step(double* state, int layout, int64_t ld, int64_t nac, const double* cmd, int substeps,
                            double fcs_dt, double* obs17, f16_stream_t stream) {
  int rc = check_state_args(state, layout, ld, nac);
  if (rc) return rc;
  if (!cmd || substeps < 1 || !(fcs_dt > 0.0)) return F16_ERR_ARG;
  if (!aligned(cmd, 16) || (obs17 && !aligned(obs17, 8))) return F16_ERR_ALIGN;
  BinGrid g{};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (layout == F16_LAYOUT_SOA)
    return launch_step<F16_LAYOUT_SOA, false>(state, ld, nac, cmd, nullptr, g, substeps, fcs_dt, obs17, s);
  return launch_step<F16_LAYOUT_AOS, false>(state, ld, nac, cmd, nullptr, g, substeps, fcs_dt, obs17, s);
}

extern "C" int f16_fdm_step_ex(double* state, int layout, int64_t ld, int64_t nac, const f16_fdm_io* io,
                               int substeps, double fcs_dt, f16_stream_t stream) {
  int rc = check_state_args(state, layout, ld, nac);
  if (rc) return rc;
  if (!io || (!io->cmd == !io->bins) || substeps < 1 || !(fcs_dt > 0.0)) return F16_ERR_ARG;
  if ((io->obs17 && !aligned(io->obs17, 8))) return F16_ERR_ALIGN;
  BinGrid g{};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (io->cmd) {
    if (!aligned(io->cmd, 16)) return F16_ERR_ALIGN;
    if (layout == F16_LAYOUT_SOA)
      return launch_step<F16_LAYOUT_SOA, false>(state, ld, nac, io->cmd, nullptr, g, substeps, fcs_dt, io->obs17, s,
                                                io->finite);
    return launch_step<F16_LAYOUT_AOS, false>(state, ld, nac, io->cmd, nullptr, g, substeps, fcs_dt, io->obs17, s,
                                              io->finite);
  }
  if (!io->grid_host || io->num_bins < 2 || io->num_bins > 64) return F16_ERR_ARG;
  if (!aligned(io->bins, 4)) return F16_ERR_ALIGN;
  for (int i = 0; i < io->num_bins; i++) {
    float v = io->grid_host[i];
    volatile float half_v = 0.5f * v;
    g.ch[i] = (double)v;
    g.thr[i] = (double)(half_v + 0.5f);
  }
  if (layout == F16_LAYOUT_SOA)
    return launch_step<F16_LAYOUT_SOA, true>(state, ld, nac, nullptr, io->bins, g, substeps, fcs_dt, io->obs17, s,
                                             io->finite);
  return launch_step<F16_LAYOUT_AOS, true>(state, ld, nac, nullptr, io->bins, g, substeps, fcs_dt, io->obs17, s,
                                           io->finite);
}

extern "C" int f16_fdm_step_bins(double* state, int layout, int64_t ld, int64_t nac, const uint8_t* bins,
                                 const float* grid_host, int num_bins, int substeps, double fcs_dt, double* obs17,
                                 f16_stream_t stream) {
  int rc = check_state_args(state, layout, ld, nac);
  if (rc) return rc;
  if (!bins || !grid_host || num_bins < 2 || num_bins > 64 || substeps < 1 || !(fcs_dt > 0.0)) return F16_ERR_ARG;
  if (!aligned(bins, 4) || (obs17 && !aligned(obs17, 8))) return F16_ERR_ALIGN;
  // channel values as the caller's float32 grid; throttle 0.5*v + 0.5 evaluated in float32
  BinGrid g{};
  for (int i = 0; i < num_bins; i++) {
    float v = grid_host[i];
    volatile float half_v = 0.5f * v;   // keep the two float32 roundings of the reference
    g.ch[i] = (double)v;
    g.thr[i] = (double)(half_v + 0.5f);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (layout == F16_LAYOUT_SOA)
    return launch_step<F16_LAYOUT_SOA, true>(state, ld, nac, nullptr, bins, g, substeps, fcs_dt, obs17, s);
  return launch_step<F16_LAYOUT_AOS, true>(state, ld, nac, nullptr, bins, g, substeps, fcs_dt, obs17, s);
}

extern "C" int f16_seed_ic(const double* ic, int64_t nac, double* state, int layout, int64_t ld, double fcs_dt,
                           f16_stream_t stream) {
  int rc = check_state_args(state, layout, ld, nac);
  if (rc) return rc;
  if (!ic || !(fcs_dt > 0.0)) return F16_ERR_ARG;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (layout == F16_LAYOUT_SOA) {
    auto k = k_seed_ic<F16_LAYOUT_SOA>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FDM_SMEM);
    k<<<persistent_grid(k, nac, FDM_SMEM), FDM_THREADS, FDM_SMEM, s>>>(ic, nac, state, ld, fcs_dt);
  } else {
    auto k = k_seed_ic<F16_LAYOUT_AOS>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)FDM_SMEM);
    k<<<persistent_grid(k, nac, FDM_SMEM), FDM_THREADS, FDM_SMEM, s>>>(ic, nac, state, ld, fcs_dt);
  }
  return launch_status();
}

extern "C" const char* f16_version(void) { return "f16env-b200 0.1 (sm_100a)"; }

extern "C" const char* f16_status_string(int status) {
  switch (status) {
    case F16_OK: return "ok";
    case F16_ERR_ARG: return "invalid argument";
    case F16_ERR_ALIGN: return "misaligned pointer";
    case F16_ERR_LAUNCH: return "kernel launch failed";
    case F16_ERR_NONFINITE: return "non-finite value detected";
    case F16_ERR_CUDA: return "CUDA runtime error";
    case F16_ERR_TOO_LARGE: return "size above the documented maximum";
    default: return "unknown status";
  }
}
