// Stand-in for leanstream_b200/csrc/ls_internal.h when ls_stream.cu is built
// against the host-only CUDA stub (test infrastructure): the engine needs only
// the public header.
#pragma once
#include <stdint.h>
#include <cuda_runtime.h>
#include "leanstream_b200.h"
