/* A plain C99 consumer of include/hymoe.h, compiled and run by tests/test_c_abi.py: the header
 * must compile as C with every warning an error, link against libhymoe.so, and the entry
 * points that need no device must behave from C as documented.  Exit status 0 = all checks
 * passed; otherwise the number of the first failing check. */
#include <math.h>
#include <stdio.h>
#include <string.h>

#include "hymoe.h"

#define CHECK(n, cond)                                   \
    do {                                                 \
        if (!(cond)) {                                   \
            fprintf(stderr, "check %d failed: %s\n", n, #cond); \
            return n;                                    \
        }                                                \
    } while (0)

int main(int argc, char** argv) {
    CHECK(1, strstr(hymoe_version(), "sm_100a") != NULL);
    /* no context: statuses, never a crash */
    CHECK(2, hymoe_create(NULL, NULL) == HYMOE_ERR_INVALID_ARG);
    CHECK(3, hymoe_forward(NULL, 0, NULL, NULL, NULL, 0, NULL, NULL, 0) == HYMOE_ERR_INVALID_ARG);
    CHECK(4, hymoe_set_routing(NULL, NULL) == HYMOE_ERR_INVALID_ARG);
    /* placement helper */
    {
        double load[64];
        int32_t slot[64];
        int seen[64] = {0};
        for (int e = 0; e < 64; ++e) load[e] = (double)((e * 37) % 64);
        CHECK(5, hymoe_balance_placement(64, 8, load, slot) == HYMOE_OK);
        for (int e = 0; e < 64; ++e) {
            CHECK(6, slot[e] >= 0 && slot[e] < 64 && !seen[slot[e]]);
            seen[slot[e]] = 1;
        }
        CHECK(7, hymoe_balance_placement(64, 3, load, slot) == HYMOE_ERR_INVALID_ARG);
    }
    /* GGUF reader on the file given as argv[1] (blk.3, 8 experts, H = 256, I = 128, Q4_0) */
    if (argc > 1) {
        hymoe_gguf* f = NULL;
        hymoe_tensor r, sgu, sdn, egu[8], edn[8];
        uint32_t v = 0;
        CHECK(8, hymoe_gguf_open(argv[1], &f) == HYMOE_OK && f != NULL);
        CHECK(9, hymoe_gguf_get_u32(f, "hunyuan.num_experts", &v) == HYMOE_OK && v == 8);
        CHECK(10, hymoe_gguf_moe_tensors(f, 3, 8, &r, &sgu, &sdn, egu, edn) == HYMOE_OK);
        CHECK(11, r.ggml_type == HYMOE_TYPE_F32 && r.ne[0] == 256 && r.ne[1] == 8);
        CHECK(12, egu[7].ggml_type == HYMOE_TYPE_Q4_0 && egu[7].ne[0] == 256 && egu[7].ne[1] == 256 &&
                      egu[7].nbytes == (size_t)256 * 256 / 32 * 18);
        CHECK(13, hymoe_gguf_tensor(f, "blk.3.missing.weight", &r) == HYMOE_ERR_INVALID_ARG);
        CHECK(14, strstr(hymoe_gguf_last_error(), "missing") != NULL);
        hymoe_gguf_close(f);
        CHECK(15, hymoe_gguf_open("/nonexistent/file.gguf", &f) == HYMOE_ERR_INVALID_ARG && f == NULL);
    }
    puts("ok");
    return 0;
}
