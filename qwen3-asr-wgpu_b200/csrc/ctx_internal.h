// Library-internal access to a context from the host-side translation units (the
// checkpoint loader): not part of the C ABI.
#pragma once
#include <string>

#include "qasr_b200.h"

namespace qasr {
// The context's text config and weight format; false for a null context.
bool ctx_shape(const qasr_ctx* c, qasr_text_config* cfg, int* weight_format);
// Record `msg` as the context's last error and return `s`.
qasr_status ctx_fail(qasr_ctx* c, qasr_status s, const std::string& msg);
}  // namespace qasr
