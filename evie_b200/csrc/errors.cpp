// Error-message storage behind evie_last_global_error().
#include "common.h"

namespace evie {
std::string& thread_error() {
  thread_local std::string msg;
  return msg;
}
}  // namespace evie

extern "C" const char* evie_last_global_error(void) { return evie::thread_error().c_str(); }
