// Matmul problem description shared by the SIMT and tensor-core GEMM paths.
#pragma once

#include "common.cuh"

namespace mtc {

constexpr int kMaxBatchRank = MTC_MAX_RANK - 2;

// C[b][m][n] = sum_k A[b][m][k] * B[b][k][n], every operand an arbitrary
// strided view (the reference MatmulPlan, src/tensor/backend/cpu/iteration/matmul.cpp:32-82).
struct GemmProblem {
    int64_t M, N, K;
    const float *A;
    const float *B;
    float *C;
    int64_t a_off, a_rs, a_cs;  // A: row (m) and column (k) strides
    int64_t b_off, b_rs, b_cs;  // B: row (k) and column (n) strides
    int64_t c_off, c_rs, c_cs;  // C: row (m) and column (n) strides
    int batch_rank;
    int64_t batch_shape[kMaxBatchRank];
    int64_t a_bs[kMaxBatchRank], b_bs[kMaxBatchRank], c_bs[kMaxBatchRank];
    int64_t batch;  // product of batch_shape
};

// tcgen05 3xTF32 path; returns MTC_ERR_UNSUPPORTED when the problem does not suit it.
int gemm_3xtf32(const GemmProblem &p, cudaStream_t stream);
// SIMT path (any strides, any sizes).  exact: the CPU reference's rounding and
// order (float product, then float sum, k ascending); otherwise one FFMA per k.
int gemm_simt(const GemmProblem &p, cudaStream_t stream, bool exact);
// The tensor-core path with its split operands in a fixed static device array
// (no allocation); rejects problems whose workspace exceeds that array.
int gemm_3xtf32_static(const GemmProblem &p, cudaStream_t stream);
// Called when the process creates a collective communicator: from then on the
// tensor-core GEMMs hand out their work units at run time, since collective
// kernels on other streams may hold some SMs while a GEMM starts.
void gemm_note_collectives();

}  // namespace mtc
