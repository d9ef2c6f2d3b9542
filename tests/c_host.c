/* A plain C99 host of libsttb200: what a non-Python caller (the Rust crate's extern "C" block,
 * a cgo or JNI stub) sees of the boundary.  Uses only calls that need no device:
 *   c_host config                      prints the default stt_config
 *   c_host load <gguf>                 loads a GGUF with the default config and prints the status and
 *                                      error text (the loader validates the whole file before it
 *                                      touches a device)
 *   c_host spm <model> <id> [<id>...]  decodes token ids with the SentencePiece detokeniser
 * Exit status 0 on success, 1 on a failed call, 2 on bad usage. */
#include <stdio.h>
#include <stdlib.h>

#include "stt_b200.h"

static unsigned char* read_file(const char* path, size_t* len) {
    FILE* f = fopen(path, "rb");
    unsigned char* buf = NULL;
    long n;
    if (!f) return NULL;
    if (fseek(f, 0, SEEK_END) != 0 || (n = ftell(f)) < 0 || fseek(f, 0, SEEK_SET) != 0) {
        fclose(f);
        return NULL;
    }
    buf = (unsigned char*)malloc(n > 0 ? (size_t)n : 1u);
    if (buf && fread(buf, 1, (size_t)n, f) != (size_t)n) {
        free(buf);
        buf = NULL;
    }
    fclose(f);
    *len = (size_t)n;
    return buf;
}

static int cmd_config(void) {
    stt_config c;
    stt_config_default(&c);
    printf("%d %d %d %d %d %d %d %d %d %d %.1f %d %d %u %u\n", c.num_layers, c.hidden_size, c.num_heads,
           c.num_kv_heads, c.intermediate_size, c.vocab_size, c.text_in_vocab_size, c.num_codebooks,
           c.audio_vocab_size, c.text_delay, c.rope_theta, c.max_seq_len, c.sliding_window, c.text_padding_id,
           c.text_start_token);
    return 0;
}

static int cmd_load(const char* path) {
    size_t len = 0;
    unsigned char* data = read_file(path, &len);
    const uint8_t* shards[1];
    stt_config c;
    stt_model* m = NULL;
    int rc;
    if (!data) return 2;
    shards[0] = data;
    stt_config_default(&c);
    rc = stt_model_load_gguf(shards, &len, 1, 0, &c, &m);
    printf("%d %s\n", rc, stt_last_error());
    free(data);
    if (m) stt_model_destroy(m);
    return 0;
}

static int cmd_spm(const char* path, int n, char** args) {
    size_t len = 0, out_len = 0;
    unsigned char* data = read_file(path, &len);
    stt_spm_decoder* d = NULL;
    uint32_t* ids;
    char* text;
    int64_t vocab = 0;
    int i;
    if (!data) return 2;
    if (stt_spm_decoder_create(data, len, &d) != STT_OK) {
        fprintf(stderr, "create: %s\n", stt_last_error());
        free(data);
        return 1;
    }
    free(data); /* the decoder keeps its own copy of the vocabulary */
    ids = (uint32_t*)malloc(sizeof(uint32_t) * (size_t)(n > 0 ? n : 1));
    for (i = 0; i < n; ++i) ids[i] = (uint32_t)strtoul(args[i], NULL, 10);
    if (stt_spm_vocab_len(d, &vocab) != STT_OK || stt_spm_decode(d, ids, (size_t)n, NULL, 0, &out_len) != STT_OK) {
        fprintf(stderr, "decode: %s\n", stt_last_error());
        return 1;
    }
    text = (char*)malloc(out_len + 1);
    if (stt_spm_decode(d, ids, (size_t)n, text, out_len + 1, &out_len) != STT_OK) {
        fprintf(stderr, "decode: %s\n", stt_last_error());
        return 1;
    }
    printf("%lld\n%s\n", (long long)vocab, text);
    free(text);
    free(ids);
    stt_spm_decoder_destroy(d);
    return 0;
}

int main(int argc, char** argv) {
    if (argc >= 2 && argv[1][0] == 'c') return cmd_config();
    if (argc == 3 && argv[1][0] == 'l') return cmd_load(argv[2]);
    if (argc >= 3 && argv[1][0] == 's') return cmd_spm(argv[2], argc - 3, argv + 3);
    fprintf(stderr, "usage: c_host config | load <gguf> | spm <model> <id>...\n");
    return 2;
}
