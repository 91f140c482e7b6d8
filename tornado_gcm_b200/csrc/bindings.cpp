// Python module entry point for the tornado_gcm_b200._C extension.  The
// operators themselves are registered with TORCH_LIBRARY_FRAGMENT(tgcm, ...)
// in the .cu files and are reached through torch.ops.tgcm.*.
#include <torch/extension.h>

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "tornado_gcm_b200 sm_100a kernels (registered under torch.ops.tgcm)";
  m.attr("arch") = "sm_100a";
}

#include <torch/library.h>

#include "alloc.h"

namespace tgcm {
namespace {
void set_poison_mode(bool on) { poison_flag() = on; }
bool poison_mode() { return poison_flag(); }
}  // namespace
}  // namespace tgcm

TORCH_LIBRARY_FRAGMENT(tgcm, m) {
  m.def("set_poison_mode(bool on) -> ()", &tgcm::set_poison_mode);
  m.def("poison_mode() -> bool", &tgcm::poison_mode);
}
