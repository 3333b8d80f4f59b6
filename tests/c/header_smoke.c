/* include/vxk.h compiles on its own as C11 (-std=c11 -Wall -Wextra -Werror
 * -pedantic); the reference checks its public headers the same way
 * (tests/headers/public_header_smoke.c). */
#include <vxk.h>

int main(void) {
    vxk_pool * pool = 0;
    vxk_enc_pool * enc = 0;
    vxk_head * head = 0;
    vxk_qweight * qw = 0;
    vxk_gguf * gguf = 0;
    vxk_decoder * dec = 0;
    vxk_encoder * encoder = 0;
    vxk_batcher * batcher = 0;
    vxk_pool_config pc = {0};
    vxk_decoder_kv_ring ring = {0};
    vxk_decoder_kv_plan plan = {0};
    vxk_enc_kv_plan eplan = {0};
    vxk_batch_fn fn = 0;
    (void) pool; (void) enc; (void) head; (void) qw; (void) gguf; (void) dec; (void) encoder;
    (void) batcher; (void) pc; (void) ring; (void) plan; (void) eplan; (void) fn;
    return VXK_STATUS_OK;
}
