/* pm_host.h - host-side helpers shared by the .cu translation units. */
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>

/* 1 on success, 0 on failure: the return convention of every pulsar_*
 * entry point (cu:25-29 cuda_ok, klib:212-218 check) */
static inline int pm_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return 1;
    fprintf(stderr, "pulsar-b200: %s: %s\n", what, cudaGetErrorString(e));
    return 0;
}

static inline int pm_cur_device() {
    int d = 0;
    cudaGetDevice(&d);
    return d;
}

/* raise a kernel's dynamic shared-memory cap to the most the device
 * allows next to the kernel's static shared memory, once per (kernel,
 * device); a request above it fails cleanly */
template <class K>
static inline int pm_smem_attr(K kernel, uint32_t bytes, uint64_t *done_mask) {
    if (bytes <= 48u * 1024u) return 1;
    const int dev = pm_cur_device();
    if (dev < 64 && (*done_mask >> dev) & 1ull) return 1;
    int optin = 0;
    cudaFuncAttributes fa;
    if (!pm_ok(cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev), "smem optin query") ||
        !pm_ok(cudaFuncGetAttributes(&fa, kernel), "kernel attributes"))
        return 0;
    const int avail = optin - (int)fa.sharedSizeBytes;
    if ((int)bytes > avail) {
        fprintf(stderr, "pulsar-b200: %u bytes of shared memory requested, kernel allows %d\n", bytes, avail);
        return 0;
    }
    if (!pm_ok(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, avail), "smem attribute")) {
        (void)cudaGetLastError();
        return 0;
    }
    if (dev < 64) *done_mask |= 1ull << dev;
    return 1;
}

/* device error word used by kernels that have no workspace argument */
uint32_t *pm_global_err_word();
