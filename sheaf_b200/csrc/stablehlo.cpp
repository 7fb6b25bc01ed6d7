// StableHLO text front door (filled in by the parser / pattern matcher).
#include "runtime.h"

namespace sb {

sb_status load_stablehlo_module(Session&, const char*, size_t, std::unique_ptr<Module>*) {
  return make_status(SB_STATUS_UNIMPLEMENTED, "StableHLO front door not built yet");
}

}  // namespace sb
