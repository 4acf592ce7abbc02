// The fused kernels with phase stamps (ls_b200_layer_args.trace): the same
// source as ls_kernel.cu, compiled with its stamp code enabled.
#define LS_KERNEL_TRACE 1
#include "ls_kernel.cu"
