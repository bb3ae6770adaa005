// C interface of the CPU checker built from the reference's kernel sources.
// Test infrastructure only (see ref_kernels.cpp).
#pragma once
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif
typedef struct xpref_arg {
    const void* ptr;   // buffer base pointer, or pointer to the POD value
    uint32_t size;     // POD size in bytes (ignored for buffers)
    int is_buffer;
} xpref_arg;
const char* xpref_last_error(void);
int xpref_find(const char* module, const char* name);
int xpref_count(void);
int xpref_kernel_info(int id, const char** module, const char** name, uint32_t* nargs,
                      int* kinds, uint32_t* sizes);
int xpref_launch(const char* module, const char* name, uint32_t grid, const xpref_arg* args,
                 uint32_t nargs, int threads);
#ifdef __cplusplus
}
#endif
