// Ring planners of the C ABI (include/vxk.h).  Pure host arithmetic with the
// semantics of the reference's planners:
//   decoder: voxtral_decoder_kv_plan / decoder_kv_commit_plan
//            (src/voxtral.cpp:1604-1656)
//   encoder: voxtral_enc_kv_plan / voxtral_enc_kv_mask_allows
//            (src/voxtral.cpp:3636-3692)
#include "vxk.h"

#include <algorithm>
#include <cstring>

namespace {

// Splits the logical span [start, start+len) of a ring into <= 2 physical
// segments in ascending-position order.
int32_t ring_segments(int64_t start, int32_t len, int32_t capacity, vxk_kv_seg out[2]) {
    if (len <= 0) return 0;
    const int32_t slot = static_cast<int32_t>(start % capacity);
    const int32_t first = std::min(len, capacity - slot);
    out[0].slot = slot;
    out[0].len = first;
    if (first == len) return 1;
    out[1].slot = 0;
    out[1].len = len - first;
    return 2;
}

}  // namespace

extern "C" {

vxk_status vxk_decoder_kv_plan_make(const vxk_decoder_kv_ring * ring, int64_t absolute_start,
                                    int32_t n_new, vxk_decoder_kv_plan * out) {
    if (!ring || !out) return VXK_STATUS_INVALID_ARGUMENT;
    std::memset(out, 0, sizeof(*out));
    const vxk_decoder_kv_ring & r = *ring;
    if (r.capacity <= 0 || r.capacity > INT32_MAX || r.used < 0 || r.used > r.capacity ||
        r.oldest_absolute_position < 0 || r.next_absolute_position < 0 ||
        r.oldest_absolute_position + r.used != r.next_absolute_position ||
        absolute_start != r.next_absolute_position || n_new <= 0 || n_new > r.capacity) {
        return VXK_STATUS_INVALID_ARGUMENT;
    }
    const int32_t cap = static_cast<int32_t>(r.capacity);
    out->absolute_start = absolute_start;
    out->n_new = n_new;
    out->write_nseg = ring_segments(absolute_start, n_new, cap, out->write_seg);
    out->next_after = absolute_start + n_new;
    out->used_after = std::min<int64_t>(r.capacity, r.used + n_new);
    out->oldest_after = out->next_after - out->used_after;
    out->evicted = std::max<int64_t>(0, r.used + n_new - r.capacity);
    out->read_nseg = ring_segments(out->oldest_after, static_cast<int32_t>(out->used_after), cap,
                                   out->read_seg);
    // A wrap is an append whose absolute span crosses a capacity cycle
    // boundary, including a single-token write landing exactly on slot 0.
    const int64_t previous_cycle = absolute_start == 0 ? 0 : (absolute_start - 1) / r.capacity;
    const int64_t newest_cycle = (out->next_after - 1) / r.capacity;
    out->wrapped = newest_cycle > previous_cycle ? 1 : 0;
    return VXK_STATUS_OK;
}

vxk_status vxk_decoder_kv_plan_commit(vxk_decoder_kv_ring * ring, const vxk_decoder_kv_plan * plan) {
    if (!ring || !plan) return VXK_STATUS_INVALID_ARGUMENT;
    ring->used = plan->used_after;
    ring->oldest_absolute_position = plan->oldest_after;
    ring->next_absolute_position = plan->next_after;
    ring->evictions += plan->evicted;
    if (plan->wrapped) ++ring->wraps;
    return VXK_STATUS_OK;
}

int32_t vxk_enc_kv_mask_allows(int64_t kv_abs, int64_t q_abs, int32_t window) {
    return (kv_abs <= q_abs && kv_abs >= q_abs - static_cast<int64_t>(window - 1)) ? 1 : 0;
}

vxk_status vxk_enc_kv_plan_make(int64_t q_start, int32_t n_new, int32_t capacity, int32_t window,
                                vxk_enc_kv_plan * out) {
    if (!out) return VXK_STATUS_INVALID_ARGUMENT;
    std::memset(out, 0, sizeof(*out));
    if (n_new <= 0 || capacity <= 0 || window <= 0) return VXK_STATUS_INVALID_ARGUMENT;
    // The ring must hold a batch's whole causal window (window-1+n_new frames)
    // so it is one logical span and the write never clobbers a live frame.
    if (n_new > capacity - window) return VXK_STATUS_INVALID_ARGUMENT;
    if (q_start < 0) return VXK_STATUS_INVALID_ARGUMENT;
    out->q_start = q_start;
    out->n_new = n_new;
    out->win_start = std::max<int64_t>(0, q_start - static_cast<int64_t>(window - 1));
    out->win_end = q_start + n_new;
    out->win_len = static_cast<int32_t>(out->win_end - out->win_start);
    out->read_nseg = ring_segments(out->win_start, out->win_len, capacity, out->read_seg);
    out->read_wraps = out->read_nseg > 1 ? 1 : 0;
    out->write_nseg = ring_segments(q_start, n_new, capacity, out->write_seg);
    out->write_wraps = out->write_nseg > 1 ? 1 : 0;
    // Even-aligned conv input with two encoder frames of real left context,
    // except at the true stream start.
    out->conv_mel_start = std::max<int64_t>(0, 2 * (q_start - 2));
    out->conv_mel_end = 2 * (q_start + n_new);
    out->conv_slice_start = static_cast<int32_t>(q_start - out->conv_mel_start / 2);
    // The cache keeps [max(0, head - window), head); evictions are the advance
    // of that lower bound over this batch.
    const int64_t old_lo = std::max<int64_t>(0, q_start - static_cast<int64_t>(window));
    const int64_t new_lo = std::max<int64_t>(0, out->win_end - static_cast<int64_t>(window));
    out->evicted = new_lo - old_lo;
    return VXK_STATUS_OK;
}

const char * vxk_status_string(vxk_status status) {
    switch (status) {
        case VXK_STATUS_OK: return "ok";
        case VXK_STATUS_INVALID_ARGUMENT: return "invalid_argument";
        case VXK_STATUS_INVALID_STATE: return "invalid_state";
        case VXK_STATUS_OUT_OF_MEMORY: return "out_of_memory";
        case VXK_STATUS_NOT_READY: return "not_ready";
        case VXK_STATUS_BACKEND_ERROR: return "backend_error";
        case VXK_STATUS_INTERNAL_ERROR: return "internal_error";
        case VXK_STATUS_BUFFER_TOO_SMALL: return "buffer_too_small";
        case VXK_STATUS_TIMEOUT: return "timeout";
        default: return "unknown";
    }
}

uint32_t vxk_api_version(void) { return VXK_API_VERSION; }

}  // extern "C"
