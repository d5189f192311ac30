/* Test support exported by librgc_b200.so beside the device ABI of rgc.h. These entry points
 * replace nothing in the reference: they let CPU tests build the row-chain kernels the device
 * generates (RGC_ROW_CHAINS=1) for a plan blob, compile them with NVRTC for sm_100a and run
 * them on the host, without a GPU or a CUDA context. */
#ifndef RGC_TEST_H
#define RGC_TEST_H

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Generates the row-chain kernels of a plan blob and compiles them without loading them.
 * Returns the number of distinct kernels, or -1 with the compiler's log in `log` (chains that
 * fall back to step-by-step lowering are listed there either way). With RGC_ROW_DUMP=<path> in
 * the environment the sources are also written to that file. */
int rgc_debug_row_kernels(const void* blob, size_t size, char* log, size_t cap);

/* Describes the kernel of row chain `index` of a plan blob as JSON in `json` (the chain's steps,
 * the slots bound to its parameters, periods, broadcast descriptors, rows, rows per block,
 * shared memory) and writes the generated-kernel prelude and its source to `source_path`.
 * Returns 0; 1 when there is no such chain or it falls back to step-by-step lowering; -1 with
 * the reason in `json`. */
int rgc_debug_row_kernel(const void* blob, size_t size, int index, char* json, size_t cap, const char* source_path);

#ifdef __cplusplus
}
#endif

#endif
