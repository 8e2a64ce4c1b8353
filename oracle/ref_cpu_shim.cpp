// ref_cpu_shim.cpp — TEST INFRASTRUCTURE. Makes the reference's own CPU check
// code callable: this translation unit includes the reference's unmodified
// tests/kernel_tests.cu (its main renamed by -Dmain=reference_kernel_tests_main)
// and exports C entry points over it. Built into oracle/_ref/libref_cpu.so with
// fake_cudart.cpp and launch_on_oracle.cpp by oracle/Makefile.
#include "kernel_tests.cu"

#include <algorithm>

// reference_rope (tests/kernel_tests.cu:175-187) on one token: out and x are
// [heads][head_dim] floats.
extern "C" void ref_reference_rope(float* out, const float* x, int seq_pos, int head_dim, int heads, double theta) {
  const std::vector<float> in(x, x + static_cast<size_t>(heads) * head_dim);
  const std::vector<float> r = reference_rope(in, seq_pos, head_dim, heads, theta);
  std::copy(r.begin(), r.end(), out);
}

// The reference's whole kernel_tests main(), with its launch_* served by the
// oracle; returns its exit status (0 = every check passed).
extern "C" int ref_kernel_tests_main(void) { return reference_kernel_tests_main(); }

// reference_gemm (tests/kernel_tests.cu:49-59): c [m][n] = a [m][k] * b [k][n], floats.
extern "C" void ref_reference_gemm(float* c, const float* a, const float* b, int m, int n, int k) {
  const std::vector<float> va(a, a + static_cast<size_t>(m) * k), vb(b, b + static_cast<size_t>(k) * n);
  const std::vector<float> r = reference_gemm(va, vb, m, n, k);
  std::copy(r.begin(), r.end(), c);
}
