// The reference library, compiled from its own source file where it lies, with
// one extra entry point: dbs_ref_force_scalar(on) pins the calling thread's
// kernel dispatch to the reference's scalar path (the path the oracle
// restates operation by operation), instead of the SIMD kernels the library
// picks at run time.
//
// TEST INFRASTRUCTURE ONLY: oracle/Makefile builds it into
// oracle/_ref/libdbs_ref_scalar.so, and tests/test_cpu_oracle_golden.py uses
// it to compare the oracle's weights and weight-dependent gradients with the
// reference's scalar arithmetic bit for bit. The product never loads it.
#include "differentiable_beam.cpp"

extern "C" DBS_EXPORT void dbs_ref_force_scalar(int on) {
    dbs::g_kernel_override_enabled = on != 0;
    dbs::g_kernel_override = dbs::KernelPath::Scalar;
}
