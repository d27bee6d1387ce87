// nnls.cu — beta fit (NNLS) and worst-key refinement.
#include "engine.h"

int kvc_launch_beta(const kvc_unit * d_units, int n_units, int max_nq, int max_t, const kvc_params_dev & P,
                    float * fs, int * is, double * gs, const kvc_layer_out * d_outs, cudaStream_t st) {
    (void)d_units; (void)n_units; (void)max_nq; (void)max_t; (void)P; (void)fs; (void)is; (void)gs;
    (void)d_outs; (void)st;
    fprintf(stderr, "[kvc] beta fit not available in this build\n");
    return KVC_ERR_SHAPE;
}

int kvc_launch_refine(const kvc_unit * d_units, int n_units, const kvc_params_dev & P, float * fs,
                      int * is, const kvc_layer_out * d_outs, cudaStream_t st) {
    (void)d_units; (void)n_units; (void)P; (void)fs; (void)is; (void)d_outs; (void)st;
    fprintf(stderr, "[kvc] refinement not available in this build\n");
    return KVC_ERR_SHAPE;
}
