/* Test helper, preloaded (LD_PRELOAD) into a child process by tests/test_zz_no_alloc.py:
 * counts the CUDA runtime calls that allocate device memory (cudaMalloc) or synchronise the
 * device through a blocking copy (cudaMemcpy) when the caller is libscx.so, and forwards
 * every call to the real runtime.  libscx.so imports both from libcudart.so.12 by dynamic
 * symbol, so a preloaded definition is the one it binds to.
 *
 *   gcc -shared -fPIC -O1 -o alloc_probe.so alloc_probe.c -ldl -Wl,--version-script=alloc_probe.map
 */
#define _GNU_SOURCE
#include <dlfcn.h>
#include <stddef.h>
#include <string.h>

typedef int (*malloc_fn)(void**, size_t);
typedef int (*memcpy_fn)(void*, const void*, size_t, int);

static int g_malloc_calls;
static int g_memcpy_calls;

static int called_from_libscx(void* ret) {
    Dl_info info;
    if (!dladdr(ret, &info) || info.dli_fname == NULL) return 0;
    return strstr(info.dli_fname, "libscx") != NULL;
}

/* The runtime's own definition.  libcudart.so.12 is usually loaded as a dependency of a
 * library opened with RTLD_LOCAL (torch, libscx.so), which RTLD_NEXT does not search, so the
 * already loaded runtime is also looked up by its soname. */
static void* real_symbol(const char* name) {
    void* f = dlvsym(RTLD_NEXT, name, "libcudart.so.12");
    if (f == NULL) f = dlsym(RTLD_NEXT, name);
    if (f == NULL) {
        void* h = dlopen("libcudart.so.12", RTLD_LAZY | RTLD_NOLOAD);
        if (h != NULL) {
            f = dlvsym(h, name, "libcudart.so.12");
            if (f == NULL) f = dlsym(h, name);
        }
    }
    return f;
}

int cudaMalloc(void** ptr, size_t bytes) {
    static malloc_fn real;
    if (real == NULL) real = (malloc_fn)real_symbol("cudaMalloc");
    if (called_from_libscx(__builtin_return_address(0))) __atomic_add_fetch(&g_malloc_calls, 1, __ATOMIC_SEQ_CST);
    return real != NULL ? real(ptr, bytes) : 999; /* 999: cudaErrorUnknown */
}

int cudaMemcpy(void* dst, const void* src, size_t bytes, int kind) {
    static memcpy_fn real;
    if (real == NULL) real = (memcpy_fn)real_symbol("cudaMemcpy");
    if (called_from_libscx(__builtin_return_address(0))) __atomic_add_fetch(&g_memcpy_calls, 1, __ATOMIC_SEQ_CST);
    return real != NULL ? real(dst, src, bytes, kind) : 999;
}

/* Calls counted so far: cudaMalloc from libscx.so, cudaMemcpy from libscx.so. */
int alloc_probe_mallocs(void) { return __atomic_load_n(&g_malloc_calls, __ATOMIC_SEQ_CST); }
int alloc_probe_memcpys(void) { return __atomic_load_n(&g_memcpy_calls, __ATOMIC_SEQ_CST); }
