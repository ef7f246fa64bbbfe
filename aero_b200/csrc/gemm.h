// Prefill grouped GEMM (tcgen05 / TMEM) entry points.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace aero {

// Device workspace the prefill path needs for P routed pairs and T tokens.
size_t gemm_workspace_bytes(int dp, int act_ld, int P, int T, int n_groups);

}  // namespace aero
