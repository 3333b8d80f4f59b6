// include/vxk.h compiles on its own as C++17 (-std=c++17 -Wall -Wextra
// -Werror -pedantic) with C linkage for every entry point; the reference
// checks its public headers the same way (tests/headers/public_header_smoke.cpp).
#include <vxk.h>

#include <type_traits>

static_assert(std::is_standard_layout<vxk_pool_config>::value, "plain C struct");
static_assert(std::is_trivially_copyable<vxk_decoder_kv_plan>::value, "plain C struct");
static_assert(sizeof(vxk_status) == sizeof(int), "status is a C enum");

int main() {
    vxk_status (*make)(const vxk_decoder_kv_ring *, int64_t, int32_t, vxk_decoder_kv_plan *) =
        &vxk_decoder_kv_plan_make;
    vxk_status (*decode)(vxk_pool *, int32_t, const float *, const float *, const float *, float *, void *) =
        &vxk_decode_layer;
    (void) make;
    (void) decode;
    vxk_pool_config pc{};
    (void) pc;
    return VXK_STATUS_OK;
}
