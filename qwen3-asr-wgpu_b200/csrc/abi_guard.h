// Host exceptions must not cross the C ABI.  The entry points whose host buffers grow
// with the caller's input or a file's contents (prefill rows, session prefixes, batch
// segments, checkpoint tensors, the page list of a context) run their body through
// guard(), which turns a failed host allocation into QASR_ERR_OOM and any other C++
// exception into QASR_ERR_STATE, each with a message for the caller's last-error slot.
#pragma once
#include <exception>
#include <new>
#include <string>

#include "qasr_b200.h"

namespace qasr {
template <class Body, class Report>
qasr_status guard(Body&& body, Report&& report) noexcept {
  try {
    return body();
  } catch (const std::bad_alloc&) {
    try {
      return report(QASR_ERR_OOM, std::string("out of host memory"));
    } catch (...) {
      return QASR_ERR_OOM;
    }
  } catch (const std::exception& e) {
    try {
      return report(QASR_ERR_STATE, std::string("host error: ") + e.what());
    } catch (...) {
      return QASR_ERR_STATE;
    }
  } catch (...) {
    try {
      return report(QASR_ERR_STATE, std::string("host error"));
    } catch (...) {
      return QASR_ERR_STATE;
    }
  }
}
}  // namespace qasr
