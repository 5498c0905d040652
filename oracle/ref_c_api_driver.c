/*
 * ref_c_api_driver.c -- runs the reference's C API test against
 * libcubutterfly_b200.so one subtest at a time (TEST INFRASTRUCTURE ONLY).
 *
 * The reference's tests/test_c_api.c is compiled unchanged: this file
 * includes it (its path comes from REF_C_API_TEST on the compiler command
 * line, see oracle/Makefile) with its `main` renamed, so its static subtests
 * can be called one by one.  The reference's own main stops at the first
 * failing subtest; here every subtest runs and reports a line
 *     SUBTEST <name> PASS|FAIL
 * on stdout (a failing subtest prints the reference's own diagnostics on
 * stderr).  Then the reference's main runs as written ("WHOLE rc=<rc>"), and
 * the number of WARNING log events seen ("WARNINGS <n>").
 */
#define main reference_c_api_main
#include REF_C_API_TEST
#undef main

typedef int (*subtest_fn)(cubutterflyHandle_t, cudaStream_t);

static int ntt_order_32_fwd(cubutterflyHandle_t h, cudaStream_t s) { return run_ntt_output_order(h, s, 32, 0, 0); }
static int ntt_order_32_inv(cubutterflyHandle_t h, cudaStream_t s) { return run_ntt_output_order(h, s, 32, 1, 0); }
static int ntt_order_64_fwd(cubutterflyHandle_t h, cudaStream_t s) { return run_ntt_output_order(h, s, 64, 0, 0); }
static int ntt_order_64_inv(cubutterflyHandle_t h, cudaStream_t s) { return run_ntt_output_order(h, s, 64, 1, 0); }
static int ntt_order_64_measure(cubutterflyHandle_t h, cudaStream_t s) { return run_ntt_output_order(h, s, 64, 0, 1); }
static int xd_u32_measure(cubutterflyHandle_t h, cudaStream_t s) { (void)s; return run_xd_uint32_ntt_measure(h); }
static int core_selection(cubutterflyHandle_t h, cudaStream_t s) { (void)s; return run_hierarchical_core_selection(h); }
static int measure_cache(cubutterflyHandle_t h, cudaStream_t s) { (void)s; return run_measure_cache(h); }
static int appt_layout(cubutterflyHandle_t h, cudaStream_t s) { (void)s; return run_appt_layout_query(h); }

static const struct {
    const char* name;
    subtest_fn fn;
} kSubtests[] = {
    {"run_2d_fwht", run_2d_fwht},
    {"run_xd_rank3_fwht", run_xd_rank3_fwht},
    {"run_embedding_fwht", run_embedding_fwht},
    {"run_strided_embedding_fwht", run_strided_embedding_fwht},
    {"run_arbitrary_fft", run_arbitrary_fft},
    {"run_2d_arbitrary_fft", run_2d_arbitrary_fft},
    {"run_2d_power_fft", run_2d_power_fft},
    {"run_2d_ntt", run_2d_ntt},
    {"run_xd_uint32_ntt_measure", xd_u32_measure},
    {"run_arbitrary_ntt", run_arbitrary_ntt},
    {"run_hierarchical_ntt", run_hierarchical_ntt},
    {"run_hierarchical_core_selection", core_selection},
    {"run_appt_layout_query", appt_layout},
    {"run_measure_cache", measure_cache},
    {"run_ntt_output_order_w32_forward", ntt_order_32_fwd},
    {"run_ntt_output_order_w32_inverse", ntt_order_32_inv},
    {"run_ntt_output_order_w64_forward", ntt_order_64_fwd},
    {"run_ntt_output_order_w64_inverse", ntt_order_64_inv},
    {"run_ntt_output_order_w64_measure", ntt_order_64_measure},
    {"run_2d_zeta", run_2d_zeta},
    {"run_2d_structured", run_2d_structured},
};

int main(int argc, char** argv) {
    cudaStream_t stream = NULL;
    cubutterflyHandle_t handle = NULL;
    int warnings = 0;
    if (cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking) != cudaSuccess ||
        cubutterflyCreate(&handle) != CUBUTTERFLY_STATUS_SUCCESS ||
        cubutterflySetStream(handle, stream) != CUBUTTERFLY_STATUS_SUCCESS ||
        cubutterflySetLogCallback(handle, log_message, &warnings) != CUBUTTERFLY_STATUS_SUCCESS) {
        fprintf(stderr, "driver set-up failed\n");
        return 2;
    }
    for (size_t i = 0; i < sizeof(kSubtests) / sizeof(kSubtests[0]); ++i) {
        const int rc = kSubtests[i].fn(handle, stream);
        fflush(stderr);
        printf("SUBTEST %s %s\n", kSubtests[i].name, rc == 0 ? "PASS" : "FAIL");
        fflush(stdout);
    }
    cubutterflyDestroy(handle);
    cudaStreamDestroy(stream);
    printf("WARNINGS %d\n", warnings);
    char* whole_argv[2] = {argv[0], NULL};
    (void)argc;
    const int whole = reference_c_api_main(1, whole_argv);
    printf("WHOLE rc=%d\n", whole);
    return 0;
}
