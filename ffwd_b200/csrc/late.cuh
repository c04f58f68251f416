// Late-interaction (ColBERT-style) device kernels: per-token vectors from the
// final hidden states and MaxSim scores.
//
// Replaces the host-side half of the reference's CUDA late path
// (libffwd/cuda.cu:5331-5452 projects on the GPU, copies every token vector to
// the host, then gathers kept rows, L2-normalises them and scores MaxSim there,
// libffwd/late.c:143-219): here the kept rows are gathered, normalised and
// scored on the device and only the vectors the caller asks for (or the
// scores) cross PCIe.  Semantics follow the CPU path the oracle checks
// (libffwd/late_blas.c:57-170): the decoder's final RMSNorm is applied to every
// token before the projection (forward.c:470-490 forwards with
// apply_final_norm = 1), the projection has no bias, the L2 norm of a zero or
// non-finite vector is an error (vec.c:7-22), and a document's score is the
// sum over query vectors of the best dot product with its kept vectors.
#pragma once

#include <cuda_runtime.h>

namespace fb {

// out[i, :] = l2norm?(W . norm?(x[rows[i], :])) for i < n_rows; W is given
// transposed, wt[h * dim + o] = W[o, h]; final_norm may be null (BERT).  A
// zero / non-finite vector under `normalize` records kErrBadNorm in err.
int late_project_launch(const float *x, int H, const int *rows, int n_rows,
                        const float *final_norm, float eps, const float *wt, int dim,
                        int normalize, float *out, int *err, cudaStream_t s);

// scores[d] = sum_{q < nq} max_{t in [doc_off[d], doc_off[d+1])} q_vec[q] . doc_vec[t]
// (vectors of length dim, row-major; doc_off[0] = 0).
int late_maxsim_launch(const float *q_vec, int nq, const float *doc_vec, const int *doc_off,
                       int n_docs, int dim, float *scores, cudaStream_t s);

// Largest token_dim the kernels take.
constexpr int kLateMaxDim = 1024;

}  // namespace fb
