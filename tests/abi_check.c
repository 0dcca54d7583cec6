/* A plain C (C11) caller of the library, as a foreign-language binding or ggml's C side would be: the header
 * compiles as C, the library links, and calls that fail validation return their status without a device.
 * Built and run by tests/test_abi.py::test_plain_c_caller. */
#include <stdio.h>
#include <string.h>

#include "klein_b200.h"

static kb_tensor tensor(int32_t type, int64_t ne0, int64_t ne1, int64_t ne2, size_t es) {
    kb_tensor t;
    memset(&t, 0, sizeof t);
    t.type = type;
    t.ne[0] = ne0, t.ne[1] = ne1, t.ne[2] = ne2, t.ne[3] = 1;
    t.nb[0] = es, t.nb[1] = es * (size_t) ne0, t.nb[2] = t.nb[1] * (size_t) ne1, t.nb[3] = t.nb[2] * (size_t) ne2;
    t.data = (void*) (uintptr_t) (1u << 20); /* never dereferenced: validation fails first */
    return t;
}

int main(void) {
    int failures = 0;
    const char* v = kb_version();
    if (!v || strncmp(v, "klein_b200", 10) != 0) {
        printf("kb_version: %s\n", v ? v : "(null)");
        ++failures;
    }
    kb_fa_params p;
    memset(&p, 0, sizeof p);
    p.scale = 1.0f / 16.0f;
    kb_tensor q = tensor(KB_TYPE_F32, 256, 4, 24, 4);
    kb_tensor k = tensor(KB_TYPE_F16, 256, 1024, 4, 2);
    kb_tensor vv = tensor(KB_TYPE_F16, 256, 1024, 4, 2);
    kb_tensor dst = tensor(KB_TYPE_F32, 256, 24, 4, 4);
    if (kb_flash_attn_ext(NULL, &k, &vv, NULL, &p, &dst, NULL, 0, NULL) != KB_ERR_ARG) {
        printf("null q not rejected\n");
        ++failures;
    }
    kb_tensor k128 = tensor(KB_TYPE_F16, 128, 1024, 4, 2);
    if (kb_flash_attn_ext(&q, &k128, &vv, NULL, &p, &dst, NULL, 0, NULL) != KB_ERR_BAD_SHAPE) {
        printf("head-dim mismatch not rejected\n");
        ++failures;
    }
    kb_tensor dst_bad = tensor(KB_TYPE_F32, 256, 23, 4, 4);
    if (kb_flash_attn_ext(&q, &k, &vv, NULL, &p, &dst_bad, NULL, 0, NULL) != KB_ERR_BAD_SHAPE) {
        printf("output shape not rejected\n");
        ++failures;
    }
    if (kb_flash_attn_ext_gated(&q, &k, &vv, NULL, &p, NULL, &dst, NULL, 0, NULL) != KB_ERR_ARG) {
        printf("gated call without a gate not rejected\n");
        ++failures;
    }
    printf("%s\n", failures ? "abi_check: FAILED" : "abi_check: ok");
    return failures ? 1 : 0;
}
