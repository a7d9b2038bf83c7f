// Internal entry of the fused attention (decode step).
#pragma once
#include <stddef.h>

// r4q_attn_decode_fused with `early`: 1 when seq_dev and every cache row before
// the new position were written before the kernel preceding this launch on the
// stream (the decode step sets positions at its start), so the K/V tiles are
// requested before griddepcontrol.wait.
int r4q_attn_decode_fused_ex(const void* qkv, long ld, const void* q_norm_w, const void* k_norm_w,
                             const void* cos_tab, const void* sin_tab, long tab_stride, float eps,
                             void* k_cache, void* v_cache, const float* k_scale, const float* v_scale, void* o,
                             long ldo, int B, int H, int Hk, int D, int max_seq, int seq_len,
                             const long long* seq_dev, int flags, int early, void* ws, size_t ws_bytes,
                             void* stream);
