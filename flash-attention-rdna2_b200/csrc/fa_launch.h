// fa_launch.h — host-side declarations shared by the kernel files and the C-ABI layer (api.cu).
#pragma once
#include <cuda_runtime.h>
#include "fable_attn.h"

namespace fa {
// kernel families (each returns FA_OK or an FA_ERR_* code; never aborts)
int fwd_simt(const FaFwdParams& p, int dtype, cudaStream_t st);
int fwd_sm100(const FaFwdParams& p, int dtype, cudaStream_t st, bool* taken);
int bwd_simt(const FaBwdParams& p, int dtype, cudaStream_t st);
int bwd_dsum(const FaBwdParams& p, int dtype, cudaStream_t st);
int bwd_sm100(const FaBwdParams& p, int dtype, cudaStream_t st, bool* taken);
int bwd_device_error(int clear);   // bits of the tensor-core backward's timed-out waits
// key-major copy of a dropout keep mask ([NH][ceil(SQ/32)][SK], bit r of word (h, qw, k) = row 32 qw + r);
// 32 x 32 blocks that no row can see under (causal, wl, wr) are not written
int dropout_mask_transpose(const unsigned int* bits, unsigned int* bits_t, int NH, int SQ, int SK, int causal,
                           int wl, int wr, cudaStream_t st);
int dec_run(const FaDecParams& p, int dtype, cudaStream_t st, const void* new_k, const void* new_v);
int combine_run(const FaCombineParams& p, cudaStream_t st);
int dec_device_error(int clear);   // bit 0: a decode pipeline wait timed out
// tensor-core split-K decode partials; *taken = false when the call is outside its envelope
int dec_tc_partial(const FaDecParams& p, int dtype, cudaStream_t st, bool* taken);
int dec_tc_device_error(int clear);
int rot_device_error(int clear);        // bit 0: a rotary position outside the cos/sin table
int fwd_simt_device_error(int clear);   // bit 0: an invalid block-table entry (paged forward)
// FABLE_ATTN_NO_PDL set: launch every kernel plainly (no programmatic dependent launch)
bool pdl_enabled();
int num_sms();
bool require_tc();   // FABLE_ATTN_REQUIRE_TC set: no CUDA-core fallback for fp16/bf16 fwd / bwd

int current_device();
// Raise the dynamic shared-memory limit of `func` to `bytes` once per device.
int ensure_smem(const void* func, int bytes, unsigned long long* done_mask);
}  // namespace fa
