/* simple_forward.c -- C API usage: the call sequence the reference sketches
 * (commented out) in Examples/simple_forward.c:10-39, as a program that
 * compiles against the pure-C header and runs on a B200.
 *
 *   gcc -std=c99 -Iinclude examples/simple_forward.c \
 *       -Lmamba-metal_b200/lib -lmamba_b200 -Wl,-rpath,mamba-metal_b200/lib
 */
#include <math.h>
#include <stdio.h>
#include <stdlib.h>

#include "mamba.h"

int main(void) {
    MambaConfig cfg = {256, 16, 4, 2, 1, MAMBA_F16}; /* d_model, d_state, d_conv, expand, n_layer, dtype */

    MambaModel *model = mamba_create(&cfg);
    if (!model) {
        fprintf(stderr, "create failed: %s\n", mamba_last_error());
        return 1;
    }
    if (mamba_init_weights_random(model, 1234) != 0) {
        fprintf(stderr, "weights: %s\n", mamba_last_error());
        return 1;
    }

    const int B = 1, L = 128, D = cfg.d_model;
    float *input = calloc((size_t)B * L * D, sizeof(float));
    float *output = calloc((size_t)B * L * D, sizeof(float));
    float *step_out = calloc((size_t)B * D, sizeof(float));
    if (!input || !output || !step_out) return 1;
    for (int i = 0; i < B * L * D; ++i) input[i] = (float)((i % 7) - 3) * 0.25f;

    if (mamba_forward(model, input, output, B, L) != 0) {
        fprintf(stderr, "forward: %s\n", mamba_last_error());
        return 1;
    }

    /* incremental: the last step output equals the forward's last position */
    MambaStateHandle *st = mamba_create_state(model, B);
    for (int t = 0; t < L; ++t)
        if (mamba_step(model, st, input + (size_t)t * D, step_out) != 0) {
            fprintf(stderr, "step: %s\n", mamba_last_error());
            return 1;
        }
    double diff = 0.0, ref = 0.0;
    for (int i = 0; i < D; ++i) {
        const double y = output[(size_t)(L - 1) * D + i];
        const double d = fabs(step_out[i] - y);
        if (d > diff) diff = d;
        if (fabs(y) > ref) ref = fabs(y);
    }
    printf("forward vs step at t=L-1: max|diff| / max|y| = %.3g\n", ref > 0 ? diff / ref : 0.0);

    mamba_destroy_state(st);
    mamba_destroy(model);
    free(input);
    free(output);
    free(step_out);
    return 0;
}
