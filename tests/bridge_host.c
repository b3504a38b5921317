/*
 * bridge_host.c -- a C host that reaches the helper the way the reference
 * binary does: through the reference's own src/minicpmo/gpu_bridge.c, which
 * dlmopen()s "<directory of this executable>/libminicpmo_gpu_helper.so" into
 * a private link-map namespace (LM_ID_NEWLM) and resolves the 19 symbols.
 * TEST CODE: oracle/Makefile links it with the unmodified gpu_bridge.c into
 * oracle/_ref/bridge_host; tests/test_gpu_bridge.py runs it.
 *
 *   bridge_host <input file> <logits output file>
 *
 * The input file (little-endian, written by the test): nine u32 -- layers,
 * hidden, heads, kv_heads, head_dim, ffn, vocab, context, tokens -- and the
 * tensor count; each tensor as u32 name length, name bytes, i32 dtype, u64
 * rows, u64 cols, u64 byte count, bytes; then the RoPE tables (f32
 * [context][head_dim/2], cos then sin) and one f32 embedding row per token.
 * The driver runs the reference host's per-operation decode
 * (qwen3_forward_embedding_runtime_cuda, qwen3.uya:1865-1918): every call is
 * one of the 19 bridge forwarders, and writes each token's logits.  It prints
 * one JSON line with the helper's stats and the decode rate of the tokens
 * after the first (host clock, every token's logits downloaded).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

typedef struct minicpmo_gpu_stats {
    uint64_t v[13];
} minicpmo_gpu_stats;

int minicpmo_gpu_context_create(unsigned int, int, void **, char *, size_t);
void minicpmo_gpu_context_destroy(void *);
int minicpmo_gpu_context_smoke(void *, char *, size_t);
int minicpmo_gpu_context_upload_tensor(void *, const char *, const void *, size_t, int, size_t, size_t, char *, size_t);
int minicpmo_gpu_context_prepare_attention(void *, size_t, size_t, size_t, char *, size_t);
int minicpmo_gpu_context_slot_upload_f32(void *, unsigned int, const float *, size_t, char *, size_t);
int minicpmo_gpu_context_slot_download_f32(void *, unsigned int, float *, size_t, char *, size_t);
int minicpmo_gpu_context_slot_matvec(void *, unsigned int, const char *, const void *, int, unsigned int, size_t, size_t,
                                     char *, size_t);
int minicpmo_gpu_context_slot_matvec2(void *, unsigned int, const char *, const void *, int, size_t, unsigned int,
                                      const char *, const void *, int, size_t, unsigned int, size_t, char *, size_t);
int minicpmo_gpu_context_slot_matvec3(void *, unsigned int, const char *, const void *, int, size_t, unsigned int,
                                      const char *, const void *, int, size_t, unsigned int, const char *, const void *,
                                      int, size_t, unsigned int, size_t, char *, size_t);
int minicpmo_gpu_context_slot_rms_norm(void *, unsigned int, unsigned int, const void *, size_t, float, char *, size_t);
int minicpmo_gpu_context_slot_head_norm(void *, unsigned int, const void *, size_t, size_t, char *, size_t);
int minicpmo_gpu_context_slot_rope(void *, unsigned int, size_t, size_t, size_t, float, float, const float *,
                                   const float *, size_t, char *, size_t);
int minicpmo_gpu_context_slot_add_inplace(void *, unsigned int, unsigned int, size_t, char *, size_t);
int minicpmo_gpu_context_slot_silu_mul(void *, unsigned int, unsigned int, unsigned int, size_t, char *, size_t);
int minicpmo_gpu_context_attention_slots(void *, unsigned int, unsigned int, unsigned int, unsigned int, size_t,
                                         size_t, size_t, size_t, size_t, size_t, char *, size_t);
void minicpmo_gpu_context_snapshot(void *, minicpmo_gpu_stats *);

typedef struct {
    char name[96];
    int dtype;
    uint64_t rows, cols, bytes;
    unsigned char *data;
} tensor;

static tensor *tensors;
static uint32_t n_tensors;
static char err[512];

static const tensor *find(const char *name) {
    uint32_t i;
    for (i = 0; i < n_tensors; ++i)
        if (strcmp(tensors[i].name, name) == 0) return &tensors[i];
    fprintf(stderr, "bridge_host: tensor %s missing\n", name);
    exit(3);
}

#define CHECK(call)                                                \
    do {                                                           \
        if (!(call)) {                                             \
            fprintf(stderr, "bridge_host: %s: %s\n", #call, err); \
            return 1;                                              \
        }                                                          \
    } while (0)

static int rd(FILE *f, void *p, size_t n) { return fread(p, 1, n, f) == n; }

int main(int argc, char **argv) {
    enum { HID, NRM, Q, K, V, CTX, AO, GATE, UP, FUS, DOWN, LOG };
    uint32_t hdr[10], l, t, i;
    FILE *f, *out;
    float *cos_t, *sin_t, *emb, *logits;
    void *h = NULL;
    minicpmo_gpu_stats st;
    if (argc != 3 || !(f = fopen(argv[1], "rb"))) return 2;
    if (!rd(f, hdr, sizeof(hdr))) return 2;
    const uint32_t layers = hdr[0], hidden = hdr[1], heads = hdr[2], kvh = hdr[3], hd = hdr[4], ffn = hdr[5],
                   vocab = hdr[6], context = hdr[7], ntok = hdr[8];
    n_tensors = hdr[9];
    tensors = (tensor *) calloc(n_tensors, sizeof(tensor));
    for (i = 0; i < n_tensors; ++i) {
        uint32_t nl;
        tensor *x = &tensors[i];
        if (!rd(f, &nl, 4) || nl >= sizeof(x->name) || !rd(f, x->name, nl) || !rd(f, &x->dtype, 4) ||
            !rd(f, &x->rows, 8) || !rd(f, &x->cols, 8) || !rd(f, &x->bytes, 8))
            return 2;
        x->data = (unsigned char *) malloc(x->bytes);
        if (!rd(f, x->data, x->bytes)) return 2;
    }
    cos_t = (float *) malloc((size_t) context * hd / 2 * 4);
    sin_t = (float *) malloc((size_t) context * hd / 2 * 4);
    emb = (float *) malloc((size_t) ntok * hidden * 4);
    logits = (float *) malloc((size_t) vocab * 4);
    if (!rd(f, cos_t, (size_t) context * hd / 2 * 4) || !rd(f, sin_t, (size_t) context * hd / 2 * 4) ||
        !rd(f, emb, (size_t) ntok * hidden * 4))
        return 2;
    fclose(f);
    if (!(out = fopen(argv[2], "wb"))) return 2;

    CHECK(minicpmo_gpu_context_create(0, 0, &h, err, sizeof(err)));
    CHECK(minicpmo_gpu_context_smoke(h, err, sizeof(err)));
    for (i = 0; i < n_tensors; ++i) {
        const tensor *x = &tensors[i];
        CHECK(minicpmo_gpu_context_upload_tensor(h, x->name, x->data, x->bytes, x->dtype, x->rows, x->cols, err,
                                                 sizeof(err)));
    }
    CHECK(minicpmo_gpu_context_prepare_attention(h, layers, context, (size_t) kvh * hd, err, sizeof(err)));
    struct timespec t0, t1;
    for (t = 0; t < ntok; ++t) {
        if (t == 1) clock_gettime(CLOCK_MONOTONIC, &t0);
        CHECK(minicpmo_gpu_context_slot_upload_f32(h, HID, emb + (size_t) t * hidden, hidden, err, sizeof(err)));
        for (l = 0; l < layers; ++l) {
            char n[16][96];
            const char *sfx[] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_q_norm", "attn_k_norm",
                                 "attn_output", "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
            const tensor *w[11];
            int j;
            for (j = 0; j < 11; ++j) {
                snprintf(n[j], sizeof(n[j]), "blk.%u.%s.weight", l, sfx[j]);
                w[j] = find(n[j]);
            }
            CHECK(minicpmo_gpu_context_slot_rms_norm(h, NRM, HID, w[0]->data, hidden, 1e-6f, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_matvec3(h, Q, w[1]->name, w[1]->data, w[1]->dtype, w[1]->rows, K, w[2]->name,
                                                    w[2]->data, w[2]->dtype, w[2]->rows, V, w[3]->name, w[3]->data,
                                                    w[3]->dtype, w[3]->rows, NRM, hidden, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_head_norm(h, Q, w[4]->data, heads, hd, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_head_norm(h, K, w[5]->data, kvh, hd, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_rope(h, Q, heads, hd, t, 1e6f, 1.0f, cos_t, sin_t, context, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_rope(h, K, kvh, hd, t, 1e6f, 1.0f, cos_t, sin_t, context, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_attention_slots(h, CTX, Q, K, V, l, t, heads, kvh, hd, context, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_matvec(h, AO, w[6]->name, w[6]->data, w[6]->dtype, CTX, w[6]->cols,
                                                   w[6]->rows, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_add_inplace(h, HID, AO, hidden, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_rms_norm(h, NRM, HID, w[7]->data, hidden, 1e-6f, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_matvec2(h, GATE, w[8]->name, w[8]->data, w[8]->dtype, w[8]->rows, UP,
                                                    w[9]->name, w[9]->data, w[9]->dtype, w[9]->rows, NRM, hidden, err,
                                                    sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_silu_mul(h, FUS, GATE, UP, ffn, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_matvec(h, DOWN, w[10]->name, w[10]->data, w[10]->dtype, FUS, w[10]->cols,
                                                   w[10]->rows, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_add_inplace(h, HID, DOWN, hidden, err, sizeof(err)));
        }
        {
            const tensor *on = find("output_norm.weight"), *ow = find("output.weight");
            CHECK(minicpmo_gpu_context_slot_rms_norm(h, NRM, HID, on->data, hidden, 1e-6f, err, sizeof(err)));
            CHECK(minicpmo_gpu_context_slot_matvec(h, LOG, ow->name, ow->data, ow->dtype, NRM, hidden, vocab, err,
                                                   sizeof(err)));
        }
        CHECK(minicpmo_gpu_context_slot_download_f32(h, LOG, logits, vocab, err, sizeof(err)));
        if (fwrite(logits, 4, vocab, out) != vocab) return 2;
    }
    clock_gettime(CLOCK_MONOTONIC, &t1);
    minicpmo_gpu_context_snapshot(h, &st);
    {
        const double s = (double) (t1.tv_sec - t0.tv_sec) + 1e-9 * (double) (t1.tv_nsec - t0.tv_nsec);
        printf("{\"native_quant_matvec_count\": %llu, \"attention_kernel_calls\": %llu, \"tok_per_s\": %.3f}\n",
               (unsigned long long) st.v[7], (unsigned long long) st.v[10], ntok > 1 && s > 0 ? (ntok - 1) / s : 0.0);
    }
    minicpmo_gpu_context_destroy(h);
    fclose(out);
    return 0;
}
