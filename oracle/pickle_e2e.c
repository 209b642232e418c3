/*
 * pickle_e2e.c - token-id driver for the reference forward pass.
 *
 * TEST INFRASTRUCTURE ONLY. Makes the calls pickle_chat_loop makes
 * (lee-muriithi-kingori/lestramanika src/pickle_host.c:433-521): mmap-load
 * the model, detect the arch, build the fast state and KV cache, prefill
 * the prompt with one pickle_fast_forward call, then greedy-decode with
 * pickle_fast_argmax one token per call. It takes token ids directly
 * because a synthetic model has no tokenizer vocabulary.
 *
 * Linked three ways (oracle/Makefile): against the unmodified reference
 * (golden run), against the hook-patched forward pass with the attention
 * block served by the CPU oracle, and with it served by the B200 shim.
 * The attach function below comes from whichever adapter is linked.
 *
 * usage: pickle_e2e <model.gguf> <out.bin> <n_gen> <dump.bin|-> <id> [<id>...]
 * out.bin: int32 n_prompt, int32 n_gen_done, int32 ids[n_gen_done],
 *          float top2_margin[n_gen_done], int32 vocab, float last_logits[vocab]
 * dump.bin (adapters that support it): per hook call
 *          int32 layer, int32 pos, float q[H*D], k[HK*D], v[HK*D] (inputs,
 *          before RoPE), float ao[H*D] (output).
 */
#include "pickle.h"
#include "pickle_fast.h"
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

int pickle_load_from_file_mmap(const char* path, pickle_model_t** out_model);

/* Provided by the linked adapter: route the attention block (or not). */
int  e2e_attach(pickle_fast_state_t* st);
void e2e_detach(void);

FILE* e2e_dump_file = NULL;

int main(int argc, char** argv) {
    if (argc < 6) {
        fprintf(stderr, "usage: %s model.gguf out.bin n_gen dump.bin|- id...\n", argv[0]);
        return 2;
    }
    const char* model_path = argv[1];
    const char* out_path = argv[2];
    int n_gen = atoi(argv[3]);
    if (strcmp(argv[4], "-") != 0) {
        e2e_dump_file = fopen(argv[4], "wb");
        if (!e2e_dump_file) { perror("dump"); return 2; }
    }
    int n_prompt = argc - 5;
    int32_t* prompt = (int32_t*)calloc((size_t)n_prompt, sizeof(int32_t));
    for (int i = 0; i < n_prompt; i++) prompt[i] = (int32_t)atoi(argv[5 + i]);

    pickle_model_t* model = NULL;
    int rc = pickle_load_from_file_mmap(model_path, &model);
    if (rc != PICKLE_OK) { fprintf(stderr, "load rc=%d\n", rc); return 1; }
    pickle_arch_t arch;
    rc = pickle_arch_detect(model, &arch);
    if (rc != PICKLE_OK) { fprintf(stderr, "arch rc=%d\n", rc); return 1; }
    pickle_fast_state_t state;
    rc = pickle_fast_state_init(model, &arch, &state);
    if (rc != PICKLE_OK) { fprintf(stderr, "state rc=%d\n", rc); return 1; }
    pickle_fast_kv_t kv;
    rc = pickle_fast_kv_alloc(&arch, &kv);
    if (rc != PICKLE_OK) { fprintf(stderr, "kv rc=%d\n", rc); return 1; }
    rc = e2e_attach(&state);
    if (rc != PICKLE_OK) { fprintf(stderr, "attach rc=%d\n", rc); return 1; }

    int VS = arch.vocab_size;
    float* logits = (float*)calloc((size_t)VS, sizeof(float));
    int32_t* ids = (int32_t*)calloc((size_t)(n_gen > 0 ? n_gen : 1), sizeof(int32_t));
    float* margins = (float*)calloc((size_t)(n_gen > 0 ? n_gen : 1), sizeof(float));
    size_t kv_pos = 0;
    rc = pickle_fast_forward(model, &arch, &state, prompt, (size_t)n_prompt, logits, &kv, &kv_pos);
    if (rc != PICKLE_OK) { fprintf(stderr, "prefill rc=%d\n", rc); return 1; }

    int done = 0;
    for (int i = 0; i < n_gen; i++) {
        int32_t next = pickle_fast_argmax(logits, (size_t)VS);
        if (next < 0) next = 0;
        float best = logits[next], second = -1e30f;
        for (int t = 0; t < VS; t++)
            if (t != next && logits[t] > second) second = logits[t];
        ids[done] = next;
        margins[done] = best - second;
        done++;
        if (kv_pos >= (size_t)arch.max_seq_len) break;
        int32_t one = next;
        rc = pickle_fast_forward(model, &arch, &state, &one, 1, logits, &kv, &kv_pos);
        if (rc != PICKLE_OK) { fprintf(stderr, "decode rc=%d at %d\n", rc, i); return 1; }
    }
    e2e_detach();

    FILE* f = fopen(out_path, "wb");
    if (!f) { perror("out"); return 2; }
    fwrite(&n_prompt, sizeof(int32_t), 1, f);
    fwrite(&done, sizeof(int32_t), 1, f);
    fwrite(ids, sizeof(int32_t), (size_t)done, f);
    fwrite(margins, sizeof(float), (size_t)done, f);
    fwrite(&VS, sizeof(int32_t), 1, f);
    fwrite(logits, sizeof(float), (size_t)VS, f);
    fclose(f);
    if (e2e_dump_file) fclose(e2e_dump_file);
    printf("pickle_e2e: prompt=%d generated=%d kv_pos=%zu\n", n_prompt, done, kv_pos);
    pickle_fast_kv_free(&kv);
    pickle_fast_state_free(&state);
    free(logits); free(ids); free(margins); free(prompt);
    return 0;
}
