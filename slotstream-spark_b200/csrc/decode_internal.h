// Internal (C++-linkage) entry of the CUDA-core fused decode layer, used by ssb_moe_decode_fused when the
// tensor-core layer (decode_tc.cu) cannot take a call's shape, and when the caller asks for it
// (SSB_DECODE_FUSED_CUDA_CORES): its results are the separate router / moe_decode_layer calls bit for bit.
#pragma once
#include <stdint.h>

int decode_fused_cuda_cores(const uint16_t* x, int64_t rows, int32_t topk, int32_t hidden, int32_t inter,
                            int32_t experts, const uint16_t* w_router, const uint16_t* sh_gate_w, const float* bias,
                            int32_t flags, int32_t layer, const int32_t* map_t, int64_t map_len,
                            const int64_t* slot_ptr_t, int64_t n_slots, const void* shared_record, float* logits_ws,
                            int32_t* out_idx, float* out_w, float* out_sh_gate, int64_t* out_base, float* h_buf,
                            float* o_buf, float* out, uint16_t* y, uint32_t* sync, int32_t* err, void* stream);
