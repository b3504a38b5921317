/*
 * ref_extract.c -- writes the reference GPU shim's embedded CUDA source
 * string (src/minicpmo/gpu_shim.c:500-979) to stdout.  TEST INFRASTRUCTURE
 * ONLY: linked against the reference shim compiled with -Dstatic= (see
 * oracle/Makefile) so that the string's symbol is visible; the output goes to
 * oracle/_ref/, which is never committed.
 */
#include <stdio.h>

extern const char *minicpmo_gpu_quant_kernel_source;

int main(void) {
    fputs(minicpmo_gpu_quant_kernel_source, stdout);
    return 0;
}
