// abi_common.h - shared host-side helpers of the C entry points (internal).
#pragma once

#include <cuda_runtime.h>

#include <algorithm>
#include <cstddef>

#include "internal.h"

namespace cg {

extern cudaStream_t g_stream;  // library stream (NULL = legacy default stream)
extern bool g_managed;         // allocate arenas with cudaMallocManaged

enum MemKind : int { MEM_DEVICE = 0, MEM_MANAGED = 1, MEM_HOST = 2 };
int mem_kind(const void *p);

// Stages host-memory arguments of one call through temporary device buffers.
struct Stage {
    struct Ent {
        void *host;
        void *dev;
        size_t bytes;
        bool copy_out;
    };
    Ent e[12];
    int n = 0;
    bool sync = false;  // a managed or host argument: finish synchronously
    int status = OK;

    ~Stage();
    void *add(const void *p, size_t bytes, bool copy_in, bool copy_out);
    template <class T>
    const T *in(const T *p, size_t count) {
        return (const T *)add(p, count * sizeof(T), true, false);
    }
    template <class T>
    T *out(T *p, size_t count) {
        return (T *)add(p, count * sizeof(T), false, true);
    }
    template <class T>
    T *inout(T *p, size_t count) {
        return (T *)add(p, count * sizeof(T), true, true);
    }
    // copy staged outputs back, synchronise if needed; returns the status
    int finish(int st);
};

void *op_scratch(size_t bytes);

}  // namespace cg
