/*
 * trainer_main.cu -- the reference's GPU trainer (train_kaggle.cu with
 * gpu_kernels.cu, the 343M model of gpu_kernels.h:17-31) run for a few steps
 * on a token file, then its weights written as a CKP1 checkpoint, the file
 * the reference's C generator loads (generate.c:49-76).
 *
 * The Makefile builds it three ways from the reference sources:
 *   trainer_ref  train_kaggle.cu + gpu_kernels.cu as they are (cuBLAS attention);
 *   trainer_gpu  gpu_kernels.cu's attention inside #ifndef ATTN_EXTERNAL and
 *                the library's attn_fwd / attn_bwd linked in;
 *   trainer_lse  as trainer_gpu, with train_kaggle.cu's B*H*T*T buffers
 *                (a_probs, s_Dbuf) shrunk and the lse-only probs mode.
 * The training step, the model, the initialisation and the optimiser are the
 * reference's own functions; this file replaces only main(), whose data path
 * (a Kaggle dataset, checkpoints under /kaggle/working) does not exist here.
 * The step below fills the batch and the learning rate as the reference's
 * loop does (train_kaggle.cu:384-414) and writes the CKP1 header and the
 * weight arena as its save_checkpoint does (train_kaggle.cu:274-281).
 *
 * usage: trainer_* <steps> <tokens.bin (uint16)> <losses.txt> [<ckp1 out>]
 */
#define main train_kaggle_main
#include TRAINER_SRC
#undef main

int main(int argc, char **argv) {
    if (argc < 4) {
        fprintf(stderr, "usage: %s <steps> <tokens.bin> <losses.txt> [<ckp1 out>]\n", argv[0]);
        return 2;
    }
    const long steps = atol(argv[1]);
    gpu_init();
    build_registry();
    long n_tokens;
    const uint16_t *toks = map_tokens(argv[2], &n_tokens);
    if (n_tokens < (long)M_ROWS + T_SIZE + 1) {
        fprintf(stderr, "token file too small (%ld tokens)\n", n_tokens);
        return 1;
    }
    d_w = dmalloc(total_params_); d_g = dmalloc(total_params_);
    d_m = dmalloc(total_params_); d_v = dmalloc(total_params_);
    CUDA_CHECK(cudaMemset(d_g, 0, (size_t)total_params_ * sizeof(float)));
    CUDA_CHECK(cudaMemset(d_m, 0, (size_t)total_params_ * sizeof(float)));
    CUDA_CHECK(cudaMemset(d_v, 0, (size_t)total_params_ * sizeof(float)));
    alloc_acts();
    init_weights();

    int *hx = (int *)malloc((size_t)M_ROWS * sizeof(int));
    int *hy = (int *)malloc((size_t)M_ROWS * sizeof(int));
    FILE *lf = fopen(argv[3], "w");
    if (!hx || !hy || !lf) { fprintf(stderr, "cannot set up the run\n"); return 1; }
    long cursor = 0;
    float loss_h = 0.0f;
    for (long step = 1; step <= steps; step++) {
        if (cursor + (long)M_ROWS + 1 >= n_tokens) cursor = 0;
        for (int b = 0; b < B_SIZE; b++)
            for (int t = 0; t < T_SIZE; t++) {
                const long idx = cursor + (long)b * T_SIZE + t;
                hx[b * T_SIZE + t] = toks[idx] % VOCAB_SIZE;
                hy[b * T_SIZE + t] = toks[idx + 1] % VOCAB_SIZE;
            }
        cursor += (long)M_ROWS;
        CUDA_CHECK(cudaMemcpy(d_x, hx, (size_t)M_ROWS * sizeof(int), cudaMemcpyHostToDevice));
        CUDA_CHECK(cudaMemcpy(d_y, hy, (size_t)M_ROWS * sizeof(int), cudaMemcpyHostToDevice));
        const float lr = (step < WARMUP) ? LR_MAX * (float)step / WARMUP : LR_MAX;
        forward();
        CUDA_CHECK(cudaMemset(d_loss, 0, sizeof(float)));
        ce_fwd_bwd(a_logits, d_y, s_dlogits, d_loss);
        backward();
        adamw_step(d_w, d_g, d_m, d_v, total_params_, lr, BETA1, BETA2, ADAM_EPS, WDECAY, (int)step);
        CUDA_CHECK(cudaMemcpy(&loss_h, d_loss, sizeof(float), cudaMemcpyDeviceToHost));
        CUDA_CHECK(cudaGetLastError());
        fprintf(lf, "%.9g\n", loss_h);
    }
    fclose(lf);

    if (argc > 4) {
        float *staging = (float *)malloc((size_t)total_params_ * sizeof(float));
        FILE *f = fopen(argv[4], "wb");
        if (!staging || !f) { fprintf(stderr, "cannot write %s\n", argv[4]); return 1; }
        int h1[8] = {CKP_MAGIC, MAX_SEQ_LEN, DIM, N_HEADS, D_FF, N_LAYERS, VOCAB_SIZE, (int)steps};
        fwrite(h1, sizeof(int), 8, f);
        write_arena(f, d_w, total_params_, staging);
        fclose(f);
        free(staging);
    }
    return 0;
}
