// evk_cuda.h — CUDA-specific additions to the evk core (not in the
// reference's evk.h): access to the stream behind a Cmd, so callers can mix
// their own kernels, NCCL collectives or graph capture with evk::ai ops.
#pragma once

namespace evk {
struct Cmd;
// The cudaStream_t (as void*) that `cmd` enqueues on.
void* cuda_stream(Cmd& cmd);
}  // namespace evk
