// Host-side helpers shared by the C ABI translation units.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <type_traits>

#include "memforge_sm100.h"
#include "mf_common.cuh"

namespace mf {

// Records `msg` as this thread's last error and returns `code`.
int fail(int code, const std::string& msg);

// Turns a pending launch error into MF_ECUDA (with the CUDA message).
int check_launch(const char* what);

// Multiprocessor count of the current device (cached per device).
int current_sm_count();

}  // namespace mf
