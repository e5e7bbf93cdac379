// Internal helpers shared by the entry-point files of libsushi_exl3_cuda.so.
#pragma once

#include "../../include/sushi_exl3.h"
#include "sx_decode.cuh"

namespace sx {

sx_status cuda_status(cudaError_t e, const char* where = "cuda");
void note_cuda_error(cudaError_t e, const char* where);
void note_detail(const char* what, const char* why);  // the text sx_last_error_detail returns
sx_status resolve_decode(const sx_decode* dec, int n, int* kind, DecParams* dp);
sx_status check_proj(const sx_proj* p, int need_experts);
bool dtype_ok(int dt);
int sm_count();

}  // namespace sx
