// engine0.cu - Stage 0 / Stage 2 (LIF + pair STDP) engine.
#include "common.h"

namespace snnb {
Engine* make_engine_stage0(const snn_config&) {
    throw Error(SNN_ERR_UNSUPPORTED, "stage0 engine not built yet");
}
}  // namespace snnb
