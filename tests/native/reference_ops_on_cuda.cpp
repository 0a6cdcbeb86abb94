// The reference's own C++ operator API (lightning_core::ops, include/lightning_core/core/ops.hpp)
// called with Device::kCUDA, routed to liblc_b200.so by
// lightining-core_b200/integration/reference_cuda_hooks.cpp, checked against the same calls with
// Device::kCPU (the reference's CPU loops, from the reference's sources built in place).
// Exit status 0 when every kCUDA result is within tolerance of the kCPU one and every kCUDA call
// went through liblc_b200.so (not the reference's CPU fallback); prints one line per op.
#include <cmath>
#include <cstdio>
#include <random>
#include <vector>

#include "lightning_core/core/ops.hpp"

extern "C" unsigned long lcReferenceHookCalls();

namespace {

using lightning_core::runtime::Device;
using lightning_core::runtime::Status;

std::vector<float> uniform(std::size_t n, unsigned seed, float lo, float hi) {
  std::mt19937 g(seed);
  std::uniform_real_distribution<float> d(lo, hi);
  std::vector<float> v(n);
  for (auto& x : v) x = d(g);
  return v;
}

// max over elements of |got - want| - (atol + rtol |want|); <= 0 means within tolerance.
double excess(const std::vector<float>& want, const std::vector<float>& got, double atol, double rtol) {
  double worst = -1e300;
  for (std::size_t i = 0; i < want.size(); ++i) {
    const double e = std::fabs(double(got[i]) - double(want[i])) - (atol + rtol * std::fabs(double(want[i])));
    if (std::isnan(e)) return INFINITY;  // a NaN anywhere fails the op
    if (e > worst) worst = e;
  }
  return worst;
}

int report(const char* name, Status cpu, Status cuda, double ex) {
  const bool ok = cpu == Status::kSuccess && cuda == Status::kSuccess && ex <= 0.0;
  std::printf("%-10s cpu=%d cuda=%d excess=%.3g %s\n", name, int(cpu), int(cuda), ex, ok ? "ok" : "FAIL");
  return ok ? 0 : 1;
}

}  // namespace

int main() {
  namespace ops = lightning_core::ops;
  int fails = 0, cuda_calls = 0;
  const unsigned long hooks0 = lcReferenceHookCalls();

  {  // vectorAdd: default policy (host buffers uploaded, output downloaded, synchronised)
    const std::size_t n = (1u << 20) + 3;
    auto a = uniform(n, 1, -1, 1), b = uniform(n, 2, -1, 1);
    std::vector<float> c0(n), c1(n);
    const Status s0 = ops::vectorAdd(a.data(), b.data(), c0.data(), n, Device::kCPU);
    const Status s1 = ops::vectorAdd(a.data(), b.data(), c1.data(), n, Device::kCUDA);
    ++cuda_calls;
    fails += report("vectorAdd", s0, s1, excess(c0, c1, 0.0, 0.0));
  }
  for (std::size_t sz : {std::size_t(256), std::size_t(1024)}) {  // matMul: SIMT and 3xTF32 paths
    auto a = uniform(sz * sz, 3, -1, 1), b = uniform(sz * sz, 4, -1, 1);
    std::vector<float> c0(sz * sz), c1(sz * sz);
    const ops::MatMulIoPolicy pol{};
    const Status s0 = ops::matMulWithPolicy(a.data(), b.data(), c0.data(), sz, sz, sz, Device::kCPU, pol);
    const Status s1 = ops::matMulWithPolicy(a.data(), b.data(), c1.data(), sz, sz, sz, Device::kCUDA, pol);
    ++cuda_calls;
    fails += report(sz == 256 ? "matMul256" : "matMul1024", s0, s1, excess(c0, c1, 1e-4, 1e-4));
  }
  {  // matrixSub (exact) and matrixDiv (the reference's CPU build uses -ffast-math: 2e-4)
    const std::size_t rows = 513, cols = 1027;
    auto a = uniform(rows * cols, 5, -2, 2), b = uniform(rows * cols, 6, 0.5f, 2);
    std::vector<float> c0(rows * cols), c1(rows * cols);
    const ops::MatrixElementwiseIoPolicy pol{};
    Status s0 = ops::matrixSubWithPolicy(a.data(), b.data(), c0.data(), rows, cols, Device::kCPU, pol);
    Status s1 = ops::matrixSubWithPolicy(a.data(), b.data(), c1.data(), rows, cols, Device::kCUDA, pol);
    ++cuda_calls;
    fails += report("matrixSub", s0, s1, excess(c0, c1, 0.0, 0.0));
    s0 = ops::matrixDivWithPolicy(a.data(), b.data(), c0.data(), rows, cols, Device::kCPU, pol);
    s1 = ops::matrixDivWithPolicy(a.data(), b.data(), c1.data(), rows, cols, Device::kCUDA, pol);
    ++cuda_calls;
    fails += report("matrixDiv", s0, s1, excess(c0, c1, 0.0, 2e-4));
  }
  const unsigned long routed = lcReferenceHookCalls() - hooks0;
  std::printf("kCUDA calls %d, served by liblc_b200.so %lu\n", cuda_calls, routed);
  if (routed != static_cast<unsigned long>(cuda_calls)) ++fails;
  return fails == 0 ? 0 : 1;
}
