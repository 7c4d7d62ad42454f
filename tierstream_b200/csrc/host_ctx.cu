// Host forward mode on CUDA (placeholder until the host-mode runtime lands): refuses the open.
#include "ctx.hpp"
#include "errors.hpp"

namespace tsb {

std::unique_ptr<HostContext> open_host_context(const Desc&, const ss_budget&, const Plan&, const ss_options&) {
  fail(SS_E_UNSUPPORTED, "ss_open: the host forward mode is not built yet in this library (use device-gated mode)");
}

}  // namespace tsb
