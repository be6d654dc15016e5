/*
 * The reference-side binding of INTEGRATION.md section 3, compiled as a C
 * program: qx_state_loop_b200 is the function a maintainer adds to
 * qx_dump_state_loop_probe_summary (src/qx_format.c:6721) for
 * --cuda-policy b200.  main() feeds it a QXF file, a prompt and a generation
 * count and prints the tokens and the cuda_profile block as JSON, so a test
 * can check the binding end to end against the CPU checker.
 *
 *   qx_state_loop_b200 <model.qxf> <ctx> <generate> <prompt token>...
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>

#include "qx_cuda.h"

static int qx_state_loop_b200(const char *qxf_path, const uint32_t *prompt, uint32_t prompt_len, uint32_t generate,
                              uint32_t ctx, uint32_t *out_tokens, FILE *json, char *err, uint64_t err_len) {
    qx_cuda_options o = {0};
    o.device = -1;                       /* current CUDA device */
    o.ctx_tokens = ctx;                  /* persistent INT8 KV capacity */
    o.flags = QX_CUDA_VERIFY_CHECKSUMS;  /* FNV of every tensor, once, like qx_verify_* */
    qx_cuda_engine *e = NULL;
    if (!qx_cuda_engine_create_from_qxf(qxf_path, &o, &e, err, err_len)) return 0;

    uint32_t next = 0, pos = prompt_len;
    /* prompt: every token at once on the tensor cores (the same result as the
       reference's one-token-at-a-time prompt loop) */
    if (!qx_cuda_prefill(e, prompt, prompt_len, 0, &next, NULL, err, err_len)) goto fail;
    /* greedy generation with the argmax fed back on the device */
    if (generate > 1 && !qx_cuda_generate(e, next, pos, generate - 1, out_tokens + 1, err, err_len)) goto fail;
    out_tokens[0] = next;

    qx_cuda_profile p;
    qx_cuda_profile_get(e, &p);
    fprintf(json, "  \"cuda_profile\": {\"enabled\": true, \"backend\": \"%s\", \"device_bytes\": %llu, "
                  "\"host_to_device_bytes\": %llu, \"device_to_host_bytes\": %llu, "
                  "\"kernel_launches\": %llu, \"graph_replays\": %llu, \"decode_steps\": %llu},\n",
            p.backend, (unsigned long long)p.device_bytes, (unsigned long long)p.host_to_device_bytes,
            (unsigned long long)p.device_to_host_bytes, (unsigned long long)p.kernel_launches,
            (unsigned long long)p.graph_replays, (unsigned long long)p.decode_steps);
    qx_cuda_engine_destroy(e);
    return 1;
fail:
    qx_cuda_engine_destroy(e);
    return 0;                            /* err already holds the message; fail-closed */
}

int main(int argc, char **argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s model.qxf ctx generate prompt_token...\n", argv[0]);
        return 2;
    }
    const uint32_t ctx = (uint32_t)strtoul(argv[2], NULL, 10), gen = (uint32_t)strtoul(argv[3], NULL, 10);
    const uint32_t np = (uint32_t)(argc - 4);
    uint32_t *prompt = calloc(np, sizeof(uint32_t)), *toks = calloc(gen ? gen : 1, sizeof(uint32_t));
    for (uint32_t i = 0; i < np; ++i) prompt[i] = (uint32_t)strtoul(argv[4 + i], NULL, 10);
    char err[512] = {0};
    printf("{\n");
    const int ok = qx_state_loop_b200(argv[1], prompt, np, gen, ctx, toks, stdout, err, sizeof err);
    if (!ok) {
        printf("  \"ok\": false, \"error\": \"%s\"\n}\n", err);
        return 1;
    }
    printf("  \"ok\": true, \"tokens\": [");
    for (uint32_t i = 0; i < gen; ++i) printf("%s%u", i ? ", " : "", toks[i]);
    printf("]\n}\n");
    free(prompt);
    free(toks);
    return 0;
}
