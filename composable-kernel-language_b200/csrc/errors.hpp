// Thread-local error message shared by every C-ABI entry point (read by ckl_last_error()).
#pragma once

#include <string>

namespace ckl {
void setLastError(const std::string &message);
}
