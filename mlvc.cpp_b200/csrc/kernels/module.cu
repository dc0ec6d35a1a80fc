// Single translation unit for the embedded sm_100a cubin: every kernel of the
// backend, resolved by name from the host through cuModuleGetFunction.
#include "sm100.cuh"

extern "C" __device__ unsigned int mlvc_b200_status = 0;
extern "C" __device__ unsigned long long mlvc_b200_wait_limit_ns = mlvc_b200::kWaitLimitNs;

#include "conv_tc.cu"
#include "ffn_tc.cu"
#include "dwconv_tc.cu"
#include "mbconv_tc.cu"
#include "bandwidth.cu"
