/* Prints the size and member offsets of pk_act and pk_kernels as whichever
 * header this is compiled against defines them: the reference's
 * backend/kernels.h (-DWITH_REFERENCE_HEADER) or this repository's
 * include/pk_kernels_abi.h. tests/test_abi.py compares the two outputs, so
 * the cuda-b200 table built against the repository's header has the
 * reference table's layout. TEST INFRASTRUCTURE ONLY. */
#ifdef WITH_REFERENCE_HEADER
#include "kernels.h"
#else
#include "pk_kernels_abi.h"
#endif
#include <stddef.h>
#include <stdio.h>

#define OFF(T, m) printf(#T "." #m " %zu\n", offsetof(T, m))

int main(void) {
    printf("pk_act %zu\n", sizeof(pk_act));
    OFF(pk_act, q); OFF(pk_act, d); OFF(pk_act, n); OFF(pk_act, qb); OFF(pk_act, T);
    printf("pk_fft %zu\n", sizeof(pk_fft));
    OFF(pk_fft, n); OFF(pk_fft, window); OFF(pk_fft, fcos); OFF(pk_fft, fsin); OFF(pk_fft, rev);
    printf("pk_kernels %zu\n", sizeof(pk_kernels));
    OFF(pk_kernels, id); OFF(pk_kernels, name); OFF(pk_kernels, needs); OFF(pk_kernels, competes);
    OFF(pk_kernels, quantize); OFF(pk_kernels, gemm_q8); OFF(pk_kernels, gemm_f32);
    OFF(pk_kernels, layernorm); OFF(pk_kernels, softmax); OFF(pk_kernels, silu);
    OFF(pk_kernels, gelu); OFF(pk_kernels, glu); OFF(pk_kernels, dwconv);
    OFF(pk_kernels, conv3x3s2); OFF(pk_kernels, lstm); OFF(pk_kernels, stft);
    OFF(pk_kernels, resample);
    return 0;
}
