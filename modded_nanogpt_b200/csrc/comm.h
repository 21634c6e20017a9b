// Peer-pointer bundle passed by value to kernels that read or write other ranks' memory over NVLink.
#pragma once
#include <stdint.h>

#define MNG_MAX_RANKS 8

typedef struct {
  void* p[MNG_MAX_RANKS];   // p[r] = address of the same buffer on rank r, as mapped in this process
  int n;                    // number of ranks (1 = local only)
  int self;                 // this rank's index into p
} PeerPtrs;
