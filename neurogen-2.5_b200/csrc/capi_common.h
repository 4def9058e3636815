// Exception-to-error-code wrappers shared by the C ABI translation units.
#pragma once
#include <exception>
#include <string>

namespace ngb {
extern thread_local std::string g_error;

template <class F> int guarded(F &&f) {
  try {
    g_error.clear();
    f();
    return 0;
  } catch (const std::exception &ex) {
    g_error = ex.what();
    return -1;
  }
}
template <class F> void *guarded_ptr(F &&f) {
  try {
    g_error.clear();
    return f();
  } catch (const std::exception &ex) {
    g_error = ex.what();
    return nullptr;
  }
}
} // namespace ngb
