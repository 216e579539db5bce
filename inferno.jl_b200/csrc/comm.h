// Internal interface of the tensor-parallel communicator (comm.cpp).
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>

struct ifr_comm;
int comm_rank(const ifr_comm *c);
int comm_world(const ifr_comm *c);
// in place: buf[0..n) = sum over ranks (no-op for one rank)
int comm_allreduce_sum(ifr_comm *c, float *buf, size_t n, cudaStream_t s);
// recv[rank][bytes] = every rank's send[bytes]
int comm_allgather_bytes(ifr_comm *c, const void *send, void *recv, size_t bytes, cudaStream_t s);
