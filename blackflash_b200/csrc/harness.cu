// Standalone correctness/benchmark harness over a gen_ref.py-style fixture
// directory. It plays the role of the reference's src/main.cu (read meta.txt and
// the raw .bin files, run, time, compare), calling the library through the
// reference-signature launcher flash_attn_naive_launch (include/flash_attn.cuh).
//
//   flash_attn <ref_dir> [iters] [peak_tflops]
//
// Differences from the reference harness:
//   * all element counts are size_t (the reference's int B*H*N*N overflows at N=65536);
//   * s_ref.bin / p_ref.bin are optional and not compared. This kernel never
//     writes S; the reference's "S debug" comparison was a development aid
//     that fails on a complete kernel by design (src/main.cu:278-297);
//   * the O check is max-abs < 0.02 against o_ref.bin, as in src/main.cu:324.
//     The l slot receives the logsumexp, and a finite-value check covers it;
//   * exit status: 0 on PASS, 1 on FAIL or any error.
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <vector>

#include "flash_attn.cuh"

#define CK(x)                                                                                   \
    do {                                                                                        \
        cudaError_t e_ = (x);                                                                   \
        if (e_ != cudaSuccess) {                                                                \
            fprintf(stderr, "CUDA error %s at %s:%d\n", cudaGetErrorString(e_), __FILE__, __LINE__); \
            return 1;                                                                           \
        }                                                                                       \
    } while (0)

static float bf16_bits_to_float(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

static bool parse_meta(const char* dir, int& B, int& H, int& N, int& d, float& scale) {
    char path[1024];
    snprintf(path, sizeof(path), "%s/meta.txt", dir);
    FILE* f = fopen(path, "r");
    if (!f) {
        fprintf(stderr, "cannot open %s\n", path);
        return false;
    }
    char line[256];
    while (fgets(line, sizeof(line), f)) {
        char key[64];
        char val[128];
        if (sscanf(line, "%63[^=]=%127s", key, val) != 2) continue;
        if (!strcmp(key, "B")) B = atoi(val);
        else if (!strcmp(key, "H")) H = atoi(val);
        else if (!strcmp(key, "N")) N = atoi(val);
        else if (!strcmp(key, "d")) d = atoi(val);
        else if (!strcmp(key, "scale")) scale = (float)atof(val);
    }
    fclose(f);
    return B > 0 && H > 0 && N > 0 && d > 0;
}

static bool load_file(const char* dir, const char* name, void* dst, size_t bytes) {
    char path[1024];
    snprintf(path, sizeof(path), "%s/%s", dir, name);
    FILE* f = fopen(path, "rb");
    if (!f) {
        fprintf(stderr, "cannot open %s\n", path);
        return false;
    }
    const size_t got = fread(dst, 1, bytes, f);
    fclose(f);
    if (got != bytes) {
        fprintf(stderr, "%s: expected %zu bytes, read %zu\n", path, bytes, got);
        return false;
    }
    return true;
}

int main(int argc, char** argv) {
    const char* dir = argc > 1 ? argv[1] : "ref_data";
    const int iters = argc > 2 ? atoi(argv[2]) : 10;
    const double peak = argc > 3 ? atof(argv[3]) : 0.0;  // optional: the device's dense bf16 TFLOP/s, for a percentage
    int B = 0, H = 0, N = 0, d = 0;
    float scale = 0.f;
    if (!parse_meta(dir, B, H, N, d, scale)) return 1;
    if (scale == 0.f) scale = 1.f / sqrtf((float)d);
    printf("BlackFlash-B200 harness: B=%d H=%d N=%d d=%d scale=%.6f dir=%s\n", B, H, N, d, scale, dir);

    const size_t n_qkv = (size_t)B * H * N * d;
    const size_t n_rows = (size_t)B * H * N;
    std::vector<uint16_t> hq(n_qkv), hk(n_qkv), hv(n_qkv), href(n_qkv), ho(n_qkv);
    if (!load_file(dir, "q.bin", hq.data(), n_qkv * 2) || !load_file(dir, "k.bin", hk.data(), n_qkv * 2) ||
        !load_file(dir, "v.bin", hv.data(), n_qkv * 2) || !load_file(dir, "o_ref.bin", href.data(), n_qkv * 2))
        return 1;

    __nv_bfloat16 *dq, *dk, *dv, *dout;
    float *dl, *dm;
    CK(cudaMalloc(&dq, n_qkv * 2));
    CK(cudaMalloc(&dk, n_qkv * 2));
    CK(cudaMalloc(&dv, n_qkv * 2));
    CK(cudaMalloc(&dout, n_qkv * 2));
    CK(cudaMalloc(&dl, n_rows * 4));
    CK(cudaMalloc(&dm, n_rows * 4));
    CK(cudaMemcpy(dq, hq.data(), n_qkv * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dk, hk.data(), n_qkv * 2, cudaMemcpyHostToDevice));
    CK(cudaMemcpy(dv, hv.data(), n_qkv * 2, cudaMemcpyHostToDevice));
    CK(cudaMemset(dout, 0, n_qkv * 2));

    blackflash_last_error();
    flash_attn_naive_launch(dq, dk, dv, dout, dl, dm, B, H, N, d, scale);
    if (blackflash_last_error()[0]) return 1;
    CK(cudaDeviceSynchronize());

    for (int i = 0; i < 3; ++i) flash_attn_naive_launch(dq, dk, dv, dout, dl, dm, B, H, N, d, scale);
    CK(cudaDeviceSynchronize());
    cudaEvent_t e0, e1;
    CK(cudaEventCreate(&e0));
    CK(cudaEventCreate(&e1));
    CK(cudaEventRecord(e0));
    for (int i = 0; i < iters; ++i) flash_attn_naive_launch(dq, dk, dv, dout, dl, dm, B, H, N, d, scale);
    CK(cudaEventRecord(e1));
    CK(cudaEventSynchronize(e1));
    float ms = 0.f;
    CK(cudaEventElapsedTime(&ms, e0, e1));
    ms /= (float)(iters > 0 ? iters : 1);
    const double fl = 4.0 * B * H * (double)N * N * d;
    const double tflops = fl / (ms * 1e-3) / 1e12;
    if (peak > 0.0)
        printf("avg latency %.4f ms, %.2f TFLOPS, %.1f%% of %.1f TFLOPS\n", ms, tflops, 100.0 * tflops / peak, peak);
    else
        printf("avg latency %.4f ms, %.2f TFLOPS\n", ms, tflops);

    CK(cudaMemcpy(ho.data(), dout, n_qkv * 2, cudaMemcpyDeviceToHost));
    std::vector<float> hl(n_rows);
    CK(cudaMemcpy(hl.data(), dl, n_rows * 4, cudaMemcpyDeviceToHost));
    double max_err = 0.0, sum_err = 0.0;
    size_t bad = 0, arg = 0;
    for (size_t i = 0; i < n_qkv; ++i) {
        const double e = fabs((double)bf16_bits_to_float(ho[i]) - (double)bf16_bits_to_float(href[i]));
        if (e > max_err) {
            max_err = e;
            arg = i;
        }
        sum_err += e;
        if (e > 0.02) ++bad;
    }
    size_t nonfinite = 0;
    for (size_t i = 0; i < n_rows; ++i) nonfinite += !isfinite(hl[i]);
    printf("O vs o_ref: max_abs %.6f (row %zu col %zu), mean_abs %.6f, %zu > 0.02, lse non-finite %zu\n", max_err,
           arg / d, arg % d, sum_err / (double)n_qkv, bad, nonfinite);
    const bool pass = max_err < 0.02 && nonfinite == 0;
    printf("Status: %s\n", pass ? "PASS" : "FAIL");
    cudaFree(dq);
    cudaFree(dk);
    cudaFree(dv);
    cudaFree(dout);
    cudaFree(dl);
    cudaFree(dm);
    return pass ? 0 : 1;
}
