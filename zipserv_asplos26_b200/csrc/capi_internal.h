// Declarations shared by the host and CUDA halves of the C ABI.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "../../include/L_API.h"

// Store a message in the thread-local channel read by zipserv_error().
void zs_set_error(const char* message);
