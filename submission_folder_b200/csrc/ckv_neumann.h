// Launch interface of the structured Neumann sweep.
#pragma once

#include <cuda_runtime.h>

#include "ckv_plan.h"

namespace ckv {

cudaError_t launch_sweep(const Plan& pl, const ckv_params& prm, char* ws, cudaStream_t st);

}  // namespace ckv
