// Process-wide switch for programmatic dependent launch (SGLANG_B200_PDL=0 turns it off, e.g. to compare).
#include <cstdlib>
#include <cstring>
#include "../common.cuh"

namespace {
int g_pdl = -1;
}

namespace snb {
bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* e = std::getenv("SGLANG_B200_PDL");
    g_pdl = (e != nullptr && (std::strcmp(e, "0") == 0 || std::strcmp(e, "false") == 0)) ? 0 : 1;
  }
  return g_pdl == 1;
}
}  // namespace snb

void set_pdl(bool on) { g_pdl = on ? 1 : 0; }
bool get_pdl() { return snb::pdl_enabled(); }
