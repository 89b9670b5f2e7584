// ref_driver.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A thin C-ABI driver around the reference's own frame step, compiled from the reference
// header where it lies (cuda_fdm/gen/fdm.cuh + f16_gen.cuh, unmodified, host-compiled the way
// the reference itself validates it: g++ -O2 -ffp-contract=off; cuda_fdm/README.md:88-99).
// oracle/build.py compiles it twice: once against the repository-root header (FCS dt 1/120,
// fdm.cuh:23) and once against research/competition_36500/runtime (FCS dt 1/60).
// The output (oracle/_ref/*.so) is the parity pin for oracle/fdm_oracle.c and the timed CPU
// baseline of bench.py --impl reference.  Nothing here is copied from the reference: the
// header is #included from its original location at build time.
#include "fdm.cuh"
#include <omp.h>

extern "C" {

// Batch step over nac aircraft, AoS (nac,101) states in place, reference FdmState order.
// The loop body is the reference's fdm_step_batch (fdm_kernel.cu:32-47) run per aircraft.
int f16ref_step(double* states, const double* cmd, long nac, int substeps, double* obs17, int nthreads) {
  if (!states || !cmd || nac < 0 || substeps < 1) return 1;
  if (nthreads > 0) omp_set_num_threads(nthreads);
#pragma omp parallel for schedule(static)
  for (long a = 0; a < nac; a++) {
    FdmState* s = reinterpret_cast<FdmState*>(states + a * 101);
    const double* c = cmd + a * 4;
    FdmOut o;
    for (int k = 0; k < substeps; k++) fdm_step(s, c[0], c[1], c[2], c[3], &o);
    if (obs17) {
      double* p = obs17 + a * 17;
      for (int i = 0; i < 3; i++) {
        p[i] = o.eci_pos[i]; p[3 + i] = o.eci_vel[i]; p[6 + i] = o.euler[i]; p[9 + i] = o.vUVW[i];
      }
      p[12] = o.alpha; p[13] = o.beta; p[14] = o.mach; p[15] = o.Vt; p[16] = o.alt_asl;
    }
  }
  return 0;
}

double f16ref_fcs_dt(void) { return FCS_DT; }
int f16ref_state_bytes(void) { return (int)sizeof(FdmState); }
int f16ref_max_threads(void) { return omp_get_max_threads(); }

}  // extern "C"
