// Drop-in check: a program written against the reference project's headers
// (gemm_kernels.h, mxfp8_utils.h, gemm_common.h) builds unchanged against this
// repository's include/ and links to libmpk.so.  The flow follows the reference's
// tests/test_gemm_correctness.cu:16-136 and tests/test_mxfp8_quantize.cu:45-102:
// seeded N(0, 0.02^2) inputs, host quantize, GPU GEMM through
// gemm_fp8_tensorcore, GPU dequantize, compare with a host FP32 gold after the
// MXFP8 round trip.  Exit code 0 on success.
#include <cstdio>
#include <random>
#include <vector>

#include "gemm_common.h"
#include "gemm_kernels.h"
#include "mxfp8_utils.h"

static bool run_gemm_case(int M, int N, int K)
{
    const int nbk = (K + MXFP8_BLOCK_SIZE - 1) / MXFP8_BLOCK_SIZE;
    const int nbn = (N + MXFP8_BLOCK_SIZE - 1) / MXFP8_BLOCK_SIZE;
    std::mt19937 rng(42);
    std::normal_distribution<float> dist(0.0f, 0.02f);
    std::vector<float> A(M * K), B(K * N), C(M * N);
    for (auto& v : A) v = dist(rng);
    for (auto& v : B) v = dist(rng);
    for (auto& v : C) v = dist(rng);

    std::vector<uint8_t> Ad(M * K), As(M * nbk), Cd(M * N), Cs(M * nbn);
    mxfp8_quantize_host(A.data(), Ad.data(), As.data(), M, K);
    mxfp8_quantize_host(C.data(), Cd.data(), Cs.data(), M, N);
    std::vector<float> Aq(M * K), Cq(M * N);
    mxfp8_dequantize_host(Ad.data(), As.data(), Aq.data(), M, K);
    mxfp8_dequantize_host(Cd.data(), Cs.data(), Cq.data(), M, N);
    std::vector<__nv_bfloat16> Bh(K * N);
    std::vector<float> Bq(K * N);
    for (int i = 0; i < K * N; ++i) {
        Bh[i] = float_to_bf16(B[i]);
        Bq[i] = bf16_to_float(Bh[i]);
    }
    // host gold: FP32 GEMM, then the MXFP8 round trip of D
    std::vector<float> Dg(M * N);
    for (int i = 0; i < M; ++i) {
        for (int j = 0; j < N; ++j) Dg[i * N + j] = 0.0f;
        for (int k = 0; k < K; ++k) {
            const float a = Aq[i * K + k];
            for (int j = 0; j < N; ++j) Dg[i * N + j] = Dg[i * N + j] + a * Bq[k * N + j];
        }
        for (int j = 0; j < N; ++j) Dg[i * N + j] = Dg[i * N + j] + Cq[i * N + j];
    }
    std::vector<uint8_t> Gd(M * N), Gs(M * nbn);
    mxfp8_quantize_host(Dg.data(), Gd.data(), Gs.data(), M, N);
    std::vector<float> Gq(M * N);
    mxfp8_dequantize_host(Gd.data(), Gs.data(), Gq.data(), M, N);

    uint8_t *dA, *dAs, *dC, *dCs, *dD, *dDs;
    __nv_bfloat16* dB;
    float* dDq;
    CUDA_CHECK(cudaMalloc(&dA, M * K));
    CUDA_CHECK(cudaMalloc(&dAs, M * nbk));
    CUDA_CHECK(cudaMalloc(&dB, K * N * sizeof(__nv_bfloat16)));
    CUDA_CHECK(cudaMalloc(&dC, M * N));
    CUDA_CHECK(cudaMalloc(&dCs, M * nbn));
    CUDA_CHECK(cudaMalloc(&dD, M * N));
    CUDA_CHECK(cudaMalloc(&dDs, M * nbn));
    CUDA_CHECK(cudaMalloc(&dDq, M * N * sizeof(float)));
    CUDA_CHECK(cudaMemcpy(dA, Ad.data(), M * K, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(dAs, As.data(), M * nbk, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(dB, Bh.data(), K * N * sizeof(__nv_bfloat16), cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(dC, Cd.data(), M * N, cudaMemcpyHostToDevice));
    CUDA_CHECK(cudaMemcpy(dCs, Cs.data(), M * nbn, cudaMemcpyHostToDevice));

    gemm_fp8_tensorcore(dA, dAs, dB, dC, dCs, dD, dDs, M, N, K);
    mxfp8_dequantize_gpu(dD, dDs, dDq, M, N);
    CUDA_CHECK(cudaDeviceSynchronize());
    std::vector<float> Dq(M * N);
    CUDA_CHECK(cudaMemcpy(Dq.data(), dDq, M * N * sizeof(float), cudaMemcpyDeviceToHost));
    const float err = compute_relative_error(Dq.data(), Gq.data(), M * N);
    const bool pass = err < 0.15f;  // tests/test_gemm_correctness.cu:150
    printf("gemm %dx%dx%d max_rel_err=%.6f %s\n", M, N, K, err, pass ? "PASS" : "FAIL");
    cudaFree(dA); cudaFree(dAs); cudaFree(dB); cudaFree(dC); cudaFree(dCs);
    cudaFree(dD); cudaFree(dDs); cudaFree(dDq);
    return pass;
}

static bool run_quantize_case(int M, int K)
{
    const int nbk = (K + MXFP8_BLOCK_SIZE - 1) / MXFP8_BLOCK_SIZE;
    std::mt19937 rng(123);
    std::uniform_real_distribution<float> dist(-5.0f, 5.0f);
    std::vector<float> x(M * K);
    for (auto& v : x) v = dist(rng);
    std::vector<uint8_t> hd(M * K), hs(M * nbk), gd(M * K), gs(M * nbk);
    mxfp8_quantize_host(x.data(), hd.data(), hs.data(), M, K);
    float* dx;
    uint8_t *dd, *ds;
    CUDA_CHECK(cudaMalloc(&dx, M * K * sizeof(float)));
    CUDA_CHECK(cudaMalloc(&dd, M * K));
    CUDA_CHECK(cudaMalloc(&ds, M * nbk));
    CUDA_CHECK(cudaMemcpy(dx, x.data(), M * K * sizeof(float), cudaMemcpyHostToDevice));
    mxfp8_quantize_gpu(dx, dd, ds, M, K);
    CUDA_CHECK(cudaDeviceSynchronize());
    CUDA_CHECK(cudaMemcpy(gd.data(), dd, M * K, cudaMemcpyDeviceToHost));
    CUDA_CHECK(cudaMemcpy(gs.data(), ds, M * nbk, cudaMemcpyDeviceToHost));
    int bad = 0;
    for (int i = 0; i < M * K; ++i) bad += gd[i] != hd[i];
    for (int i = 0; i < M * nbk; ++i) bad += gs[i] != hs[i];
    printf("quantize %dx%d gpu-vs-host mismatches=%d %s\n", M, K, bad, bad ? "FAIL" : "PASS");
    cudaFree(dx); cudaFree(dd); cudaFree(ds);
    return bad == 0;
}

int main()
{
    bool ok = true;
    ok &= run_quantize_case(128, 256);
    ok &= run_quantize_case(512, 1024);
    ok &= run_quantize_case(128, 100);
    ok &= run_gemm_case(128, 128, 128);
    ok &= run_gemm_case(256, 512, 1024);
    ok &= run_gemm_case(200, 264, 80);
    printf(ok ? "ALL PASS\n" : "FAILURES\n");
    return ok ? 0 : 1;
}
