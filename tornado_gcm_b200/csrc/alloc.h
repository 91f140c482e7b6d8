// Output / scratch allocation for the host-side op wrappers.
//
// Poison mode (environment TGCM_POISON=1, or torch.ops.tgcm.set_poison_mode)
// fills every buffer an op allocates with NaN (floating types) or all-ones
// bits (integer types) before the kernels run.  A kernel that reads an
// element before writing it then produces NaN / garbage that the numerics
// tests catch, which stands in for a race / uninitialised-read checker.
#pragma once

#include <ATen/ATen.h>

#include <cmath>
#include <cstdlib>
#include <cstring>

namespace tgcm {

inline bool& poison_flag() {
  static bool flag = [] {
    const char* v = std::getenv("TGCM_POISON");
    return v != nullptr && std::strcmp(v, "0") != 0 && v[0] != '\0';
  }();
  return flag;
}

inline at::Tensor poisoned(at::Tensor t) {
  if (poison_flag()) {
    if (t.is_floating_point())
      t.fill_(NAN);
    else
      t.fill_(-1);
  }
  return t;
}

inline at::Tensor out_empty(at::IntArrayRef sizes, const at::TensorOptions& opt) {
  return poisoned(at::empty(sizes, opt));
}

inline at::Tensor out_empty_like(const at::Tensor& x) { return poisoned(at::empty_like(x)); }

}  // namespace tgcm
