// Launch policy shared by all kernels.
#include <cstdlib>
#include <cstring>

namespace vmc {

// Programmatic dependent launch is on unless VMC_PDL=0.
bool pdl_enabled() {
  static const bool on = [] {
    const char* e = std::getenv("VMC_PDL");
    return !(e && std::strcmp(e, "0") == 0);
  }();
  return on;
}

}  // namespace vmc
