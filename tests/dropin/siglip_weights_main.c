/*
 * siglip_weights_main.c -- runs the reference's own SigLIP encoder (siglip_forward,
 * common/vision/siglip.c of tmzt/smol-genius) on weights and images read from a file
 * and writes the encoder output of every image.
 *
 * The CPU test of the SigLIP oracle (tests/test_siglip_oracle.py) writes the file from
 * the oracle's seeded weights, runs this program and compares.  oracle/Makefile links
 * it with the reference's kernel sources (attention, conv2d, layernorm, matmul,
 * activation, ...) as they lie.
 *
 * Input (little-endian): "SGLP", int32 hidden, heads, ffn_dim, layers, patch, image
 * size, num_positions, n_images; float32 layer_norm_eps; float32 patch_weight
 * [hidden][3*patch*patch], patch_bias[hidden], position_embedding[num_positions][hidden];
 * per layer float32 ln1_w, ln1_b, wq, bq, wk, bk, wv, bv, wo, bo, ln2_w, ln2_b,
 * fc1 [ffn][hidden], b1, fc2 [hidden][ffn], b2; post_ln_w, post_ln_b; images
 * [n_images][3][size][size].
 * Output: per image float32 [n_patches][hidden].
 *
 * Usage: siglip_weights_ref <in> <out>
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "siglip.h"
#include "smol_kernels.h"

static FILE *g_in;

static float *take(size_t n)
{
    float *p = (float *)malloc(sizeof(float) * (n ? n : 1));
    if (!p || fread(p, sizeof(float), n, g_in) != n) {
        fprintf(stderr, "short read\n");
        exit(2);
    }
    return p;
}

int main(int argc, char **argv)
{
    if (argc != 3) return 2;
    g_in = fopen(argv[1], "rb");
    FILE *out = fopen(argv[2], "wb");
    if (!g_in || !out) return 2;
    char magic[4];
    int32_t h[8];
    float eps;
    if (fread(magic, 1, 4, g_in) != 4 || memcmp(magic, "SGLP", 4) || fread(h, 4, 8, g_in) != 8 ||
        fread(&eps, 4, 1, g_in) != 1)
        return 2;
    const int H = h[0], F = h[2], L = h[3], P = h[4], S = h[5], NPOS = h[6], NI = h[7];
    if (L < 1 || L > SIGLIP_MAX_LAYERS) return 2;

    siglip_config_t cfg = {0};
    cfg.hidden = H;
    cfg.heads = h[1];
    cfg.head_dim = H / h[1];
    cfg.ffn_dim = F;
    cfg.image_size = S;
    cfg.patch_size = P;
    cfg.layers = L;
    cfg.layer_norm_eps = eps;

    siglip_encoder_t *enc = (siglip_encoder_t *)calloc(1, sizeof(siglip_encoder_t));
    enc->patch_weight = take((size_t)H * 3 * P * P);
    enc->patch_bias = take((size_t)H);
    enc->position_embedding = take((size_t)NPOS * H);
    enc->num_positions = NPOS;
    for (int l = 0; l < L; l++) {
        siglip_layer_t *ly = &enc->layers[l];
        ly->ln1_weight = take(H);
        ly->ln1_bias = take(H);
        ly->wq_weight = take((size_t)H * H);
        ly->wq_bias = take(H);
        ly->wk_weight = take((size_t)H * H);
        ly->wk_bias = take(H);
        ly->wv_weight = take((size_t)H * H);
        ly->wv_bias = take(H);
        ly->wo_weight = take((size_t)H * H);
        ly->wo_bias = take(H);
        ly->ln2_weight = take(H);
        ly->ln2_bias = take(H);
        ly->fc1_weight = take((size_t)F * H);
        ly->fc1_bias = take(F);
        ly->fc2_weight = take((size_t)H * F);
        ly->fc2_bias = take(H);
    }
    enc->post_ln_weight = take(H);
    enc->post_ln_bias = take(H);
    const size_t img_n = (size_t)3 * S * S;
    float *images = take(img_n * NI);
    fclose(g_in);

    int threads = smol_get_num_cpus();
    smol_set_threads(threads > 16 ? 16 : threads);
    for (int i = 0; i < NI; i++) {
        int seq = 0;
        float *y = siglip_forward(enc, &cfg, images + img_n * i, 3, S, S, &seq);
        if (!y) return 3;
        fwrite(y, sizeof(float), (size_t)seq * H, out);
        free(y);
    }
    fclose(out);
    return 0;
}
