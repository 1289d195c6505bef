/* A plain C99 caller of libspmgpu.so: the header must compile as C and the
 * host-only entry points must work through it (what a Rust `extern "C"`
 * crate or any other FFI binds).  Built and run by tests/test_c_abi.py. */
#include <stdio.h>
#include <string.h>

#include "spmgpu.h"

static int fails = 0;
#define CHECK(cond)                                                   \
    do {                                                              \
        if (!(cond)) {                                                \
            fprintf(stderr, "FAILED %s:%d %s\n", __FILE__, __LINE__, #cond); \
            fails++;                                                  \
        }                                                             \
    } while (0)

int main(void) {
    /* the 74-byte ternary file of the reference's golden test, field by field */
    static const unsigned char tiny[74] = {
        0x89, 'S', 'P', 'M', 0x0D, 0x0A, 0x1A, 0x0A, 1, 0, 0, 0, 0, 0, 0, 0, 1, 0, 0, 0,
        0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0,
        3, 0, 0, 0, 2, 0, 0, 0, 4, 0, 0, 0, 1, 0, 1, 0,
        0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0, 0,
        0x00, 0x00, 0x80, 0x3F, 0x71,
        0x00, 0x00, 0x00, 0x3F, 0x03};
    uint32_t major = 0, minor = 9;
    int32_t streams = 0;
    spm_file_stream_info info;
    uint64_t regions[3] = {256, 512, 256};
    int32_t script[4] = {SPM_PLAN_NEXT, SPM_PLAN_NEXT, SPM_PLAN_NEXT, SPM_PLAN_REWIND};
    int64_t log[4 * 64];
    int64_t records = 0;
    /* a Q8_0 block: d = 1.0, q = -16..15 */
    unsigned char q8[34];
    float out[32];
    int i;

    CHECK(spm_version() != NULL && strlen(spm_version()) > 0);
    CHECK(spm_file_probe(tiny, sizeof tiny, &major, &minor, &streams) == SPM_OK);
    CHECK(major == 1 && minor == 0 && streams == 1);
    CHECK(spm_file_stream(tiny, sizeof tiny, 0, &info) == SPM_OK);
    CHECK(info.rows == 3 && info.cols == 2 && info.group_size == 4 && info.encoding == 1);
    CHECK(info.groups == 2 && info.offset == 64 && info.bytes == 10);
    CHECK(spm_file_stream(tiny, sizeof tiny - 1, 0, &info) == SPM_E_TRUNCATED);
    CHECK(strstr(spm_last_error(), "group needs 5 bytes, 4 remain") != NULL);

    CHECK(spm_sweep_plan(regions, 3, 768, script, 4, log, 64, &records) == SPM_OK);
    CHECK(records > 0 && log[0] == SPM_PLAN_EVENTS);

    q8[0] = 0x00;
    q8[1] = 0x3C;
    for (i = 0; i < 32; ++i) q8[2 + i] = (unsigned char)(signed char)(i - 16);
    CHECK(spm_decode_blocks(SPM_Q8_0, q8, sizeof q8, out) == SPM_OK);
    for (i = 0; i < 32; ++i) CHECK(out[i] == (float)(i - 16));
    CHECK(spm_decode_blocks(SPM_Q8_0, q8, sizeof q8 - 1, out) != SPM_OK);

    if (fails) return 1;
    printf("c abi ok\n");
    return 0;
}
