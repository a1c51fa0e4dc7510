// Internal interface between the C-ABI core (ms_api.cu) and the file loader
// (ms_loader.cu).  Nothing here is exported from the library.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "../../include/mojostream_cuda.h"

// Record a failure in the context's last-error message and return s.
ms_status ms_fail_(ms_ctx* c, ms_status s, const char* msg);
cudaStream_t ms_stream_(ms_ctx* c);
int ms_device_(const ms_ctx* c);
// Device-resident BOS embedding: token id `bos_id` embeds as bos (hidden
// floats, device) instead of its lm_head column.
ms_status ms_model_set_bos_(ms_ctx* c, ms_model* m, const float* bos, int bos_id);
void ms_set_load_stats_(ms_ctx* c, double seconds, uint64_t bytes);
