// Library-wide C-ABI entry points: version, last error, PDL switch.
#include <cstdlib>
#include <cstring>
#include <string>

#include "afb_launch.h"

namespace afb {

namespace {
thread_local std::string g_last_error;
int g_pdl = -1;  // -1: read AFB_PDL from the environment on first use
}  // namespace

void set_error(const std::string& msg) { g_last_error = msg; }
const std::string& last_error() { return g_last_error; }

bool pdl_enabled() {
  if (g_pdl < 0) {
    const char* env = std::getenv("AFB_PDL");
    g_pdl = (env != nullptr && std::strcmp(env, "0") == 0) ? 0 : 1;
  }
  return g_pdl != 0;
}

}  // namespace afb

extern "C" int afb_abi_version(void) { return 1; }

extern "C" const char* afb_last_error(void) { return afb::g_last_error.c_str(); }

extern "C" void afb_clear_error(void) { afb::g_last_error.clear(); }

extern "C" void afb_set_pdl(int enabled) { afb::g_pdl = enabled ? 1 : 0; }

extern "C" int afb_get_pdl(void) { return afb::pdl_enabled() ? 1 : 0; }
