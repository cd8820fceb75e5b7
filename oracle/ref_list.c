/* The backend list for the reference's own checks (tests/q8check.c,
 * tests/kcheck.c), rebuilt by oracle/Makefile against the cuda-b200 table.
 * TEST INFRASTRUCTURE ONLY.
 *
 * The reference's checks walk pk_kernels_built (backend/kernels.h:284-285)
 * and hold every entry before ref to ref's bits (tests/q8check.c:165,
 * tests/kcheck.c:585-600). Its own list (backend/kernels.c:23-63) names
 * only CPU backends, so oracle/Makefile compiles that file with its list
 * renamed away and links this one in its place: cuda-b200, cuda-b200-f32
 * (its gemm_f32 and softmax on the GPU too: kcheck's float-product and
 * softmax cases), then ref. No reference source is modified. */
#include "kernels.h"

#include <stddef.h>

extern const pk_kernels pk_kernels_cuda_b200, pk_kernels_cuda_b200_f32;

const pk_kernels *const pk_kernels_built[] = { &pk_kernels_cuda_b200, &pk_kernels_cuda_b200_f32, &pk_kernels_ref,
                                               NULL };
