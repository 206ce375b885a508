/*
 * TEST INFRASTRUCTURE ONLY -- never linked into the product library.
 *
 * Single-node stand-in for the libnuma API subset used by the reference CPU
 * engine (Int8-gemm/numa_threadpool.h:65-76, Int8-gemm/moe_common.cpp:57-142,
 * Int8-gemm/moe_infer.cpp:11-84).  Node 0 owns every online CPU and memory
 * comes from the ordinary heap, so the reference runs unmodified on a host
 * without libnuma with NANOVLLM_TP_SIZE=1.
 */
#pragma once
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

struct bitmask {
    unsigned long size;   /* number of bits */
    unsigned long* maskp;
};

static inline int numa_available(void) { return 0; }
static inline int numa_max_node(void) { return 0; }

static inline void* numa_alloc_onnode(size_t size, int node) {
    (void)node;
    void* p = NULL;
    if (posix_memalign(&p, 4096, size ? size : 1) != 0) return NULL;
    return p;
}
static inline void numa_free(void* p, size_t size) { (void)size; free(p); }
static inline int numa_run_on_node(int node) { (void)node; return 0; }

static inline struct bitmask* numa_allocate_cpumask(void) {
    struct bitmask* bm = (struct bitmask*)calloc(1, sizeof(struct bitmask));
    long ncpu = sysconf(_SC_NPROCESSORS_ONLN);
    if (ncpu < 1) ncpu = 1;
    bm->size = (unsigned long)ncpu;
    bm->maskp = (unsigned long*)calloc((ncpu + 63) / 64, sizeof(unsigned long));
    return bm;
}
static inline void numa_free_cpumask(struct bitmask* bm) {
    if (!bm) return;
    free(bm->maskp);
    free(bm);
}
static inline int numa_node_to_cpus(int node, struct bitmask* bm) {
    if (node != 0) return -1;
    for (unsigned long c = 0; c < bm->size; ++c) bm->maskp[c / 64] |= 1ul << (c % 64);
    return 0;
}
static inline int numa_bitmask_isbitset(const struct bitmask* bm, unsigned int n) {
    if (n >= bm->size) return 0;
    return (int)((bm->maskp[n / 64] >> (n % 64)) & 1ul);
}
