// Peer-pointer bundle passed by value to kernels that read or write other ranks' memory over NVLink.
#pragma once
#include <stdint.h>

#define MNG_MAX_RANKS 8

typedef struct {
  void* p[MNG_MAX_RANKS];   // p[r] = address of the same buffer on rank r, as mapped in this process
  int n;                    // number of ranks (1 = local only)
  int self;                 // this rank's index into p
  void* mc;                 // NVSwitch multicast address of the same buffer (one access reaches every rank), or null:
                            // loads through it come back summed over the ranks, stores land on all of them
} PeerPtrs;
