/* A plain C99 caller of libtierk.so: compiled by tests/test_abi.py with
 * gcc -std=c99 -pedantic -Werror against include/tierk.h, linked to the built
 * library and run without a GPU.  It exercises the host-only entry points the
 * way a C engine would bind them and prints one line per check. */
#include <stdio.h>
#include <string.h>

#include "tierk.h"

static const int types[] = {TK_F32,    TK_F16,    TK_BF16,   TK_Q4_0,   TK_Q4_1,   TK_Q5_0,   TK_Q5_1,
                            TK_Q8_0,   TK_Q2_K,   TK_Q3_K,   TK_Q4_K,   TK_Q5_K,   TK_Q6_K,   TK_IQ4_NL,
                            TK_IQ4_XS, TK_TQ1_0,  TK_TQ2_0,  TK_MXFP4,  TK_NF4,    TK_FP4,    TK_IQ2_XXS,
                            TK_IQ2_XS, TK_IQ2_S,  TK_IQ3_XXS, TK_IQ3_S, TK_IQ1_S,  TK_IQ1_M};

int main(void) {
    size_t i;
    tk_ctx *ctx = NULL;
    tk_status st;
    for (i = 0; i < sizeof types / sizeof types[0]; ++i) {
        const char *name = tk_qtype_name(types[i]);
        printf("type %d %s %zu %d\n", types[i], name ? name : "?", tk_row_bytes(types[i], 4096),
               name ? tk_qtype_from_name(name) : -1);
    }
    st = tk_dequant(NULL, TK_Q8_0, NULL, 0, 0, 1, 32, TK_DT_F32, NULL, NULL);
    printf("null_ctx %d %d\n", (int)st, strstr(tk_last_error_string(), "null context") != NULL);
    st = tk_set_iq_grids(NULL, NULL);
    printf("null_grids %d\n", (int)st);
    st = tk_init(0, &ctx);
    printf("init %d %d\n", (int)st, ctx == NULL);
    if (ctx) tk_destroy(ctx);
    return 0;
}
