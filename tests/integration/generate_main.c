/*
 * generate_main.c -- the reference's C generator (generate.c) decoding from a
 * CKP1 checkpoint with greedy sampling, writing every step's logits.
 *
 * The Makefile builds it twice from the reference sources: as generate.c is
 * (the CPU attention loop of block(), generate.c:129-152), and with that
 * loop replaced by attn_cached_attention_host_ex (the maintainer's edit;
 * the edited copy lives in a temporary directory during the build).  The
 * model loader, the decoder block, the forward pass and the sampler are
 * generate.c's own; this file replaces only main(), which needs a BPE vocab
 * and a prompt string: here the prompt is a list of token ids.
 *
 * usage: generate_* <ckp1> <n_new> <logits out> <prompt token ids...>
 */
#define main generate_cli_main
#include GENERATE_SRC
#undef main

int main(int argc, char **argv) {
    if (argc < 5) {
        fprintf(stderr, "usage: %s <ckp1> <n_new> <logits out> <prompt token ids...>\n", argv[0]);
        return 2;
    }
    load_model(argv[1]);
    alloc_state();
    const int n_new = atoi(argv[2]);
    FILE *f = fopen(argv[3], "wb");
    if (!f) die("cannot open the logits file");
    int pos = 0, tok = 0;
    /* the prompt fills the KV cache; its last token's logits pick the first new token */
    for (int i = 4; i < argc && pos < BLK; i++, pos++) {
        tok = atoi(argv[i]);
        forward(tok < V ? tok : 0, pos);
    }
    for (int s = 0; s < n_new && pos < BLK; s++, pos++) {
        fwrite(s_logits, sizeof(float), (size_t)V, f);
        tok = sample(s_logits, V, 0.0f, 0);           /* temp 0: greedy argmax */
        forward(tok, pos);
    }
    fclose(f);
    return 0;
}
