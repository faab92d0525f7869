/* A C11 caller of libplamo_cuda compiled against include/plamo.h and include/plamo_kernels.h, as a
 * Swift/C/C++ host of the library would be. It runs without a GPU: it checks that every header
 * compiles as strict C11 (and as C++ through the same source), then calls the host-side entry
 * points and the error paths a caller hits before any device work: argument validation,
 * plamo_last_error, null-handle tolerance, the .p12 block codec and offset-chain rule
 * (Packed.swift:63-89), and Sampler.repetitionPeriod (Sampler.swift:35-51). Exit status 0 means
 * every check held; a failing check prints its line. */
#include "plamo.h"
#include "plamo_kernels.h"

#include <stdio.h>
#include <string.h>

static int failures = 0;
#define EXPECT(cond)                                                        \
    do {                                                                    \
        if (!(cond)) {                                                      \
            fprintf(stderr, "abi_caller.c:%d: check failed: %s\n", __LINE__, #cond); \
            failures++;                                                     \
        }                                                                   \
    } while (0)

int main(int argc, char** argv) {
    const char* model_dir = argc > 1 ? argv[1] : ".";
    plamo_runtime* rt = (plamo_runtime*)&failures; /* must be cleared by a failed open */

    /* plamo_open: context is validated first (Runtime.swift:164-172), then the device */
    EXPECT(plamo_open(model_dir, 0, 0, 0, &rt) != 0);
    EXPECT(rt == NULL);
    EXPECT(strstr(plamo_last_error(), "Context") != NULL);
    EXPECT(plamo_open(model_dir, 32769, 0, 0, &rt) != 0);
    EXPECT(plamo_open(model_dir, 64, 0, 0, NULL) != 0);
    /* without a CUDA device (or with one): a missing model directory never yields a handle */
    rt = (plamo_runtime*)&failures;
    EXPECT(plamo_open("/nonexistent/plamo-model", 64, 0, 0, &rt) != 0);
    EXPECT(rt == NULL);
    EXPECT(strlen(plamo_last_error()) > 0);

    /* null handles: queries return neutral values, closes and resets are no-ops */
    EXPECT(plamo_position(NULL) == 0);
    EXPECT(plamo_gpu_seconds(NULL) == 0.0);
    EXPECT(plamo_weight_bytes(NULL) == 0);
    EXPECT(plamo_device_bytes(NULL) == 0);
    EXPECT(plamo_persistent_decode(NULL) == 0);
    plamo_reset(NULL);
    plamo_close(NULL);
    plamo_batch_reset(NULL);
    plamo_batch_close(NULL);
    {
        int32_t next = 7;
        const int32_t ids[1] = {1};
        EXPECT(plamo_forward(NULL, ids, 1, 1, &next) != 0);
        EXPECT(plamo_prefill(NULL, ids, 1, &next) != 0);
        EXPECT(strstr(plamo_last_error(), "context") != NULL);
        EXPECT(plamo_set_tensor_gemm(NULL, 1) != 0);
        EXPECT(plamo_debug_wait_timeout(NULL, 1000000ull) != 0);
        plamo_batch* b = (plamo_batch*)&failures;
        EXPECT(plamo_batch_open(NULL, 4, &b) != 0);
    }

    /* Sampler.repetitionPeriod: a 2-token loop repeated 12 times (24 tokens) has period 2 */
    {
        int32_t t[40];
        for (int i = 0; i < 16; i++) t[i] = 100 + i;
        for (int i = 16; i < 40; i++) t[i] = (i & 1) ? 5 : 9;
        EXPECT(plamo_repetition_period(t, 40, 2) == 2);
        EXPECT(plamo_repetition_period(t, 40, 1) == 0);
        EXPECT(plamo_repetition_period(t, 20, 2) == 0);
        EXPECT(plamo_repetition_period(NULL, 0, 2) == 0);
    }

    /* the .p12 offset chain: packed blocks take 192 bytes, raw blocks (tag 0) 256 */
    {
        const uint32_t chain[3] = {0u | 5u, 192u | 0u, 448u | 1u};
        EXPECT(plamo_p12_chain_valid(chain, 3, 640) == 1);
        EXPECT(plamo_p12_chain_valid(chain, 3, 641) == 0);
        EXPECT(plamo_p12_chain_valid(chain, 3, 639) == 0);
        const uint32_t gap[2] = {0u | 5u, 256u | 5u};
        EXPECT(plamo_p12_chain_valid(gap, 2, 448) == 0);
        EXPECT(plamo_p12_chain_valid(chain, 0, 0) == 1);
    }

    /* the block codec: 128 weights with exponents in one packable range pack to 192 bytes whose
     * table entry carries a nonzero tag; a block spanning a wide exponent range stays raw (256) */
    {
        uint16_t v[256];
        uint8_t data[512];
        uint32_t entries[2];
        size_t used = 0;
        for (int i = 0; i < 128; i++) v[i] = (uint16_t)(((120 + (i % 10)) << 7) | (i & 127) | ((i & 1) << 15));
        for (int i = 128; i < 256; i++) v[i] = (uint16_t)(((i & 1) ? 200 : 100) << 7);
        EXPECT(plamo_pack_blocks(v, 256, data, sizeof data, entries, &used) == 0);
        EXPECT(used == 192 + 256);
        EXPECT((entries[0] & 63u) != 0 && (entries[0] & ~63u) == 0);
        EXPECT((entries[1] & 63u) == 0 && (entries[1] & ~63u) == 192);
        EXPECT(plamo_p12_chain_valid(entries, 2, used) == 1);
        EXPECT(plamo_pack_blocks(v, 100, data, sizeof data, entries, &used) != 0); /* not a multiple of 128 */
    }

    /* kernel-level entry points validate their arguments before touching a device */
    EXPECT(plamo_k_linear(NULL, NULL, NULL, 1, 128, 1, 0, NULL, NULL, NULL) != 0);
    EXPECT(strstr(plamo_last_error(), "Invalid linear arguments") != NULL);
    EXPECT(plamo_k_attention_static(NULL, NULL, NULL, 16, 1, 64, 0, 64, 0, 64, 1, NULL, 4, NULL, NULL) != 0);
    EXPECT(strstr(plamo_last_error(), "Invalid attention arguments") != NULL);
    {
        /* the multi-row attention takes tensor 0 (CUDA cores), 1 (prefill, tcgen05) or 2 (decode rows,
         * warp-level MMAs); anything else is refused before a device is touched */
        uint16_t buf[64];
        const int32_t geo[4] = {0, 64, 0, 64};
        EXPECT(plamo_k_attention_rows(buf, buf, buf, 16, 1, 64, geo, 1, 1, NULL, 4, 3, buf, buf, sizeof buf, NULL) != 0);
        EXPECT(strstr(plamo_last_error(), "Invalid attention arguments") != NULL);
    }

    if (failures) fprintf(stderr, "%d check(s) failed\n", failures);
    else printf("abi_caller: ok\n");
    return failures ? 1 : 0;
}
