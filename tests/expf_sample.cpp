// Compares jal::libm::expf_ref (the product's expf evaluation, host build)
// with the host libm expf on every `stride`-th float with |x| <= 110 plus
// special values.  Prints "checked N mismatched M" and exits non-zero on a
// mismatch.  Built and run by tests/test_libm_expf.py.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <cstdint>

#include "libm_expf.h"

static bool same(float a, float b) {
  uint32_t x, y;
  memcpy(&x, &a, 4);
  memcpy(&y, &b, 4);
  return x == y || (std::isnan(a) && std::isnan(b));
}

int main(int argc, char **argv) {
  const uint64_t stride = argc > 1 ? strtoull(argv[1], nullptr, 10) : 97;
  uint64_t n = 0, bad = 0;
  auto check = [&](float x) {
    n++;
    const float a = expf(x), b = jal::libm::expf_ref(x);
    if (!same(a, b)) {
      if (bad < 10) printf("mismatch x=%a libm=%a ref=%a\n", x, a, b);
      bad++;
    }
  };
  for (uint64_t u = 0; u < (1ull << 32); u += stride) {
    float x;
    const uint32_t b = (uint32_t)u;
    memcpy(&x, &b, 4);
    if (std::fabs(x) <= 110.0f) check(x);
  }
  const float special[] = {0.0f, -0.0f, 1.0f, -1.0f, 88.0f, -88.0f, 88.72283172607421875f, 88.7228394f,
                           -103.972076416015625f, -103.97208f, -104.0f, 1e-30f, -1e-30f, 0x1.04845ep+5f,
                           -0x1.f8cbb2p+5f, INFINITY, -INFINITY, NAN};
  for (float x : special) check(x);
  printf("checked %llu mismatched %llu\n", (unsigned long long)n, (unsigned long long)bad);
  return bad != 0;
}
