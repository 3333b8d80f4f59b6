/* A C11 program linked against libvxk.so that calls the host-only entry
 * points of include/vxk.h (no GPU needed):
 *  - the decoder ring planner, replaying the expectations of the reference's
 *    own tests/cpp/test_decoder_kv.cpp:47-115 (contiguous append, a
 *    straddled write with its logical read order, 25 single-token steps in
 *    capacity 8 with 3 wraps and 17 evictions, the invalid plans);
 *  - the encoder ring planner on tests/cpp/test_encoder_kv.cpp's first batch
 *    and overflow guards (window 750, capacity 878);
 *  - status strings, the API version, default configs, and a pool create
 *    that must fail with a status (not a crash) when no sm_100a GPU is usable.
 * Prints "ok <checks>" and exits 0, or prints the failing line and exits 1.
 * Built and run by tests/test_c_abi.py. */
#include <vxk.h>

#include <stdio.h>
#include <string.h>

static int g_checks = 0;
static int g_failed = 0;

#define CHECK(cond)                                                   \
    do {                                                              \
        ++g_checks;                                                   \
        if (!(cond)) {                                                \
            printf("FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);    \
            ++g_failed;                                               \
        }                                                             \
    } while (0)

static vxk_decoder_kv_ring ring_of(int64_t cap) {
    vxk_decoder_kv_ring r;
    memset(&r, 0, sizeof(r));
    r.capacity = cap;
    return r;
}

/* Absolute position held by each logical read index of a plan. */
static int logical_positions(const vxk_decoder_kv_plan * p, int64_t cap, int64_t * out) {
    int n = 0;
    for (int s = 0; s < p->read_nseg; ++s) {
        for (int i = 0; i < p->read_seg[s].len; ++i) {
            const int64_t slot = p->read_seg[s].slot + i;
            for (int64_t a = p->oldest_after; a < p->next_after; ++a) {
                if (a % cap == slot) {
                    out[n++] = a;
                    break;
                }
            }
        }
    }
    return n;
}

static void test_initial_and_contiguous(void) {
    vxk_decoder_kv_ring r = ring_of(8);
    vxk_decoder_kv_plan p;
    CHECK(vxk_decoder_kv_plan_make(&r, 0, 3, &p) == VXK_STATUS_OK);
    CHECK(p.write_nseg == 1 && p.write_seg[0].slot == 0 && p.write_seg[0].len == 3);
    CHECK(p.read_nseg == 1 && p.read_seg[0].slot == 0 && p.read_seg[0].len == 3);
    CHECK(p.used_after == 3 && p.oldest_after == 0 && p.next_after == 3);
    CHECK(p.evicted == 0 && !p.wrapped);
    CHECK(vxk_decoder_kv_plan_commit(&r, &p) == VXK_STATUS_OK);
    CHECK(r.used == 3 && r.next_absolute_position == 3);
}

static void test_straddled_write_and_logical_read(void) {
    vxk_decoder_kv_ring r = ring_of(8);
    vxk_decoder_kv_plan p;
    int64_t logical[16];
    int n, i;
    r.used = 6;
    r.next_absolute_position = 6;
    CHECK(vxk_decoder_kv_plan_make(&r, 6, 4, &p) == VXK_STATUS_OK);
    CHECK(p.write_nseg == 2);
    CHECK(p.write_seg[0].slot == 6 && p.write_seg[0].len == 2);
    CHECK(p.write_seg[1].slot == 0 && p.write_seg[1].len == 2);
    CHECK(p.used_after == 8 && p.oldest_after == 2 && p.next_after == 10);
    CHECK(p.evicted == 2 && p.wrapped);
    CHECK(p.read_nseg == 2);
    CHECK(p.read_seg[0].slot == 2 && p.read_seg[0].len == 6);
    CHECK(p.read_seg[1].slot == 0 && p.read_seg[1].len == 2);
    n = logical_positions(&p, 8, logical);
    CHECK(n == 8);
    for (i = 0; i < n; ++i) CHECK(logical[i] == (int64_t) i + 2);
}

static void test_single_step_rollover_and_eviction(void) {
    vxk_decoder_kv_ring r = ring_of(8);
    int64_t physical[8];
    int64_t logical[16];
    int64_t pos;
    int i, n;
    for (i = 0; i < 8; ++i) physical[i] = -1;
    for (pos = 0; pos < 25; ++pos) {
        vxk_decoder_kv_plan p;
        CHECK(vxk_decoder_kv_plan_make(&r, pos, 1, &p) == VXK_STATUS_OK);
        physical[p.write_seg[0].slot] = pos;
        CHECK(vxk_decoder_kv_plan_commit(&r, &p) == VXK_STATUS_OK);
        CHECK(r.next_absolute_position == pos + 1);
        CHECK(r.used == (pos < 7 ? pos + 1 : 8));
        CHECK(r.oldest_absolute_position == (pos < 8 ? 0 : pos - 7));
        n = logical_positions(&p, 8, logical);
        CHECK(n == r.used);
        for (i = 0; i < n; ++i) {
            CHECK(logical[i] == r.oldest_absolute_position + i);
            CHECK(physical[logical[i] % 8] == logical[i]);
        }
    }
    CHECK(r.wraps == 3);      /* writes at absolute 8, 16, 24 */
    CHECK(r.evictions == 17); /* 25 appended into capacity 8 */
    CHECK(r.bytes_moved == 0 && r.full_buffer_moves == 0);
    CHECK(r.oldest_absolute_position == 17);
}

static void test_invalid_plans(void) {
    vxk_decoder_kv_ring r = ring_of(8);
    vxk_decoder_kv_plan p;
    CHECK(vxk_decoder_kv_plan_make(&r, 1, 1, &p) != VXK_STATUS_OK); /* discontinuity */
    CHECK(vxk_decoder_kv_plan_make(&r, 0, 0, &p) != VXK_STATUS_OK);
    CHECK(vxk_decoder_kv_plan_make(&r, 0, 9, &p) != VXK_STATUS_OK);
    r.used = 2; /* inconsistent: oldest + used != next */
    CHECK(vxk_decoder_kv_plan_make(&r, 0, 1, &p) != VXK_STATUS_OK);
    CHECK(vxk_decoder_kv_plan_make(NULL, 0, 1, &p) == VXK_STATUS_INVALID_ARGUMENT);
}

static void test_encoder_plans(void) {
    vxk_enc_kv_plan p;
    const int32_t win = 750, cap = 878, max_new = cap - win;
    CHECK(vxk_enc_kv_plan_make(0, 0, cap, win, &p) != VXK_STATUS_OK);
    CHECK(vxk_enc_kv_plan_make(0, -3, cap, win, &p) != VXK_STATUS_OK);
    CHECK(vxk_enc_kv_plan_make(0, max_new + 1, cap, win, &p) != VXK_STATUS_OK);
    CHECK(vxk_enc_kv_plan_make(-1, 4, cap, win, &p) != VXK_STATUS_OK);
    CHECK(vxk_enc_kv_plan_make(0, max_new, cap, win, &p) == VXK_STATUS_OK);
    CHECK(vxk_enc_kv_plan_make(0, 1, cap, win, &p) == VXK_STATUS_OK);
    CHECK(vxk_enc_kv_plan_make(0, 4, cap, win, &p) == VXK_STATUS_OK);
    CHECK(p.win_start == 0 && p.win_end == 4 && p.win_len == 4);
    CHECK(!p.read_wraps && !p.write_wraps);
    CHECK(p.read_seg[0].slot == 0 && p.read_seg[0].len == 4);
    CHECK(p.conv_mel_start == 0 && p.conv_mel_end == 8 && p.conv_slice_start == 0);
    CHECK(p.evicted == 0);
    CHECK(vxk_enc_kv_mask_allows(0, 749, win) == 1);
    CHECK(vxk_enc_kv_mask_allows(0, 750, win) == 0);
    CHECK(vxk_enc_kv_mask_allows(751, 750, win) == 0);
}

static void test_misc(void) {
    char buf[256];
    vxk_pool_config pc = vxk_pool_default_config();
    vxk_pool * pool = NULL;
    vxk_status st;
    CHECK(strcmp(vxk_status_string(VXK_STATUS_OK), "ok") == 0);
    CHECK(strcmp(vxk_status_string(VXK_STATUS_TIMEOUT), "timeout") == 0);
    CHECK(vxk_api_version() == VXK_API_VERSION);
    CHECK(pc.struct_size == sizeof(vxk_pool_config) && pc.api_version == VXK_API_VERSION);
    CHECK(pc.n_layers == 26 && pc.n_q_heads == 32 && pc.n_kv_heads == 8 && pc.head_dim == 128);
    CHECK(pc.block_tokens == 16 && pc.capacity == 8192 && pc.dtype == VXK_DTYPE_F16 && pc.split_pages == 0);
    /* a config struct that is too short for the first published version */
    pc.struct_size = 8;
    CHECK(vxk_pool_create(&pc, &pool) == VXK_STATUS_INVALID_ARGUMENT && pool == NULL);
    pc = vxk_pool_default_config();
    pc.head_dim = 64;
    CHECK(vxk_pool_create(&pc, &pool) == VXK_STATUS_INVALID_ARGUMENT && pool == NULL);
    CHECK(vxk_pool_last_error(NULL, buf, sizeof(buf)) == VXK_STATUS_OK && strlen(buf) > 0);
    /* without a usable GPU the pool is refused with a status, never a crash */
    pc = vxk_pool_default_config();
    st = vxk_pool_create(&pc, &pool);
    if (st == VXK_STATUS_OK) {
        vxk_pool_destroy(pool);
    } else {
        CHECK(pool == NULL);
        CHECK(vxk_pool_last_error(NULL, buf, sizeof(buf)) == VXK_STATUS_OK && strlen(buf) > 0);
    }
    vxk_pool_destroy(NULL);
}

int main(void) {
    test_initial_and_contiguous();
    test_straddled_write_and_logical_read();
    test_single_step_rollover_and_eviction();
    test_invalid_plans();
    test_encoder_plans();
    test_misc();
    if (g_failed) {
        printf("failed %d of %d\n", g_failed, g_checks);
        return 1;
    }
    printf("ok %d\n", g_checks);
    return 0;
}
