/* Appended (by the Makefile) to the generated _ref/kcpu.c, after the reference's own multi-token
 * matmul section (kernels.c:1836-1913, matmul_quant_cpu and its block dequantisers): an exported
 * entry to that static function, so the checkers can run the reference's CPU prefill matmul.
 * TEST INFRASTRUCTURE ONLY. */
void ref_matmul_q(int is_q6, const void *matrix, const float *X, float *Y, size_t rows, size_t cols, size_t T)
{
    matmul_quant_cpu(is_q6, matrix, X, Y, rows, cols, T);
}
