// Matrix-product problem description shared by the tensor-core and CUDA-core
// kernels.  Strides are in elements; `c` has unit column stride.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace tpb {

struct GemmProblem {
    int dtype;
    int64_t M, N, K, batch;
    const void* a;  // A[b][m][k] at a + b*sa_b + m*sa_m + k*sa_k
    int64_t sa_b, sa_m, sa_k;
    const void* b;  // B[b][k][n] at b + b*sb_b + k*sb_k + n*sb_n
    int64_t sb_b, sb_k, sb_n;
    void* c;        // C[b][m][n] at c + b*sc_b + m*sc_m + n
    int64_t sc_b, sc_m;
    const void* cin;  // optional addend, any strides (0 = broadcast)
    int64_t sci_b, sci_m, sci_n;
    double alpha, beta;
    int flags;
    // Fused epilogue (tp_b200_gemm_epilogue): 0 none, 1 gelu (aux receives
    // the pre-activation), 2 gelu_backward (aux holds the activation's
    // input).  aux: [M x N], unit column stride, row stride saux_m.
    int epi;
    void* aux;
    int64_t saux_m;
};

void gemm_simt(const GemmProblem& p, int dev, cudaStream_t stream);
// False when the problem does not fit the tensor-core kernel's constraints
// (dtype, TMA alignment); nothing has been launched then.
bool gemm_tc(const GemmProblem& p, int dev, cudaStream_t stream);

}  // namespace tpb
