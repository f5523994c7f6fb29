// Single translation unit of the library, so that the device watchdog word
// (g_device_error) is shared by every kernel without relocatable device code.
#include "capi.cu"
#include "rep_fused.cu"
#include "quant.cu"
#include "gemm_tc.cu"
#include "moe.cu"
#include "peer.cu"
