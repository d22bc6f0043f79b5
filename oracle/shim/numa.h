/* Stub libnuma for compiling the reference's memory.cpp on a host without the
 * libnuma headers (oracle/_ref build only).  Reports "NUMA not available", so
 * nnml_memory falls back to one aligned_alloc buffer set (memory.cpp:402-446). */
#pragma once
#include <stddef.h>
#include <stdlib.h>
struct bitmask { unsigned long size; unsigned long * maskp; };
static inline int numa_available(void) { return -1; }
static inline int numa_max_node(void) { return 0; }
static inline void * numa_alloc_onnode(size_t size, int node) { (void)node; return malloc(size); }
static inline void numa_free(void * p, size_t size) { (void)size; free(p); }
static inline struct bitmask * numa_allocate_cpumask(void) { return NULL; }
static inline void numa_free_cpumask(struct bitmask * b) { (void)b; }
static inline int numa_node_to_cpus(int node, struct bitmask * b) { (void)node; (void)b; return -1; }
static inline int numa_bitmask_isbitset(const struct bitmask * b, unsigned int n) { (void)b; (void)n; return 0; }
