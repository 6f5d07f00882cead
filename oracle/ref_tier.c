/* ref_tier.c - the reference's own kernel-table self-test and tier matrix,
 * run on the CUDA tier (oracle/tlm_kern_cuda.c over libtlmg).
 *
 * TEST INFRASTRUCTURE ONLY. The reference's src/lib/tlm_quant.c and
 * tests/test_quant.c are compiled in place through the #includes below
 * (nothing is copied), which makes their static parts reachable:
 *
 *   1. selftest_tier (src/lib/tlm_quant.c:1014-1056), the check build_tier
 *      runs on every SIMD tier at start-up, on a table filled by
 *      tlm_kern_cuda_fill, against the scalar table: every entry that does
 *      not reproduce the scalar bits on the fixed data counts a failure.
 *   2. test_tiers_bitexact and test_matvec_tiles (tests/test_quant.c:
 *      708-864), with the test's tier 1 ("avx2") replaced by the CUDA table:
 *      the test's own single-row dots over every integer format, width and
 *      edge pattern, the float paths, and 8-row matvec tiles with padded
 *      strides, unaligned bases and sub-ranges, each compared bit for bit
 *      with the scalar tier.
 *
 * Prints one line per part; exits 0 when every check passed, 1 on a
 * failure, 77 when no sm_100 device is present.
 */
#define TLM_QUANT_INTERNAL 1
#include "tlm_quant.c"

int tlm_kern_cuda_fill(tlm_quant_kernels *k);

static tlm_quant_kernels g_cuda;
static int g_cuda_tier = -1;            /* test tier index served by the CUDA table */
static char g_forced[32];

/* The test selects a tier with tlm_cpu_force(name) + tlm_quant_init(); both
 * calls in tests/test_quant.c are routed here so that forcing tier
 * g_cuda_tier's name installs the CUDA table as the active one. */
static void tier_force(const char *name) {
    snprintf(g_forced, sizeof g_forced, "%s", name);
    tlm_cpu_force(!strcmp(name, "avx2") && g_cuda_tier == 1 ? "scalar" : name);
}
static void tier_init(void) {
    tlm_quant_init();
    if (g_cuda_tier == 1 && !strcmp(g_forced, "avx2"))
        atomic_store_explicit(&g_kern, (const tlm_quant_kernels *)&g_cuda, memory_order_release);
}

#define main tlm_test_quant_main
#define f2u tq_f2u            /* the test's own helpers of the same name as tlm_quant.c's */
#define u2f tq_u2f
#define tlm_cpu_force tier_force
#define tlm_quant_init tier_init
#include "tests/test_quant.c"
#undef tlm_quant_init
#undef tlm_cpu_force
#undef u2f
#undef f2u
#undef main

int main(void) {
    tlm_quant_init();
    build_tier(0);
    g_cuda = g_tab[0];
    int filled = tlm_kern_cuda_fill(&g_cuda);
    if (filled <= 0) {
        printf("cuda tier: absent (no sm_100 device)\n");
        return 77;
    }
    g_cuda.name = "cuda";
    int before = tlm_quant_selftest_failures();
    selftest_tier(&g_cuda, &g_tab[0]);
    int st_fail = tlm_quant_selftest_failures() - before;
    printf("selftest_tier cuda: %d entries filled, %d failed\n", filled, st_fail);

    g_cuda_tier = 1;
    (void)tier_ok(0);     /* the test's tier probe: scalar always, tier 2 as the CPU allows */
    g_tier_ok[1] = 1;     /* tier 1 is the CUDA table */
    RUN(test_tiers_bitexact);
    RUN(test_matvec_tiles);
    g_cuda_tier = -1;
    tlm_cpu_force("auto");
    tlm_quant_init();
    printf("tier matrix cuda: %d failure(s)\n", tlm_test_failures);
    return st_fail || tlm_test_failures ? 1 : 0;
}
