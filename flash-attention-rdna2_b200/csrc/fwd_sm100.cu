// fwd_sm100.cu — tcgen05 forward (being written; declines every request for now).
#include "fa_common.cuh"
#include "fa_launch.h"
namespace fa {
int fwd_sm100(const FaFwdParams&, int, cudaStream_t, bool* taken) { *taken = false; return FA_OK; }
}
