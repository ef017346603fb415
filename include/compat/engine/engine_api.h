// The reference's engine header name (gpu-engine/include/engine/engine_api.h), mapped onto this library's
// Engine: put include/compat on the include path ahead of gpu-engine/include and GpuEngineGenerator builds unchanged.
#include "../../b2_engine_api.hpp"
