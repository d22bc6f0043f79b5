/* Stub <numaif.h> for the oracle/_ref build (see numa.h). */
#pragma once
#define MPOL_F_NODE (1 << 0)
#define MPOL_F_ADDR (1 << 1)
static inline long get_mempolicy(int * mode, unsigned long * nodemask, unsigned long maxnode, void * addr, unsigned long flags) {
    (void)nodemask; (void)maxnode; (void)addr; (void)flags; if (mode) *mode = 0; return -1;
}
