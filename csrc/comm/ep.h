// Host entry points of the expert-parallel all-to-all kernels (csrc/comm/ep_a2a.cu).
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace bwn {

constexpr int kEpMaxRanks = 8;
// flag slots (unsigned) in each rank's flag array: [A: counts][B: rows][C: returns], W each
constexpr int kEpFlagA = 0, kEpFlagB = kEpMaxRanks, kEpFlagC = 2 * kEpMaxRanks;

struct EpArgs {
  int world, rank, e_local, H, k;
  int T;                 // this rank's tokens this call (<= T_max)
  int T_max;             // capacity of the combine buffer
  int max_recv;          // capacity of the receive buffer (rows)
  // this rank's inputs
  const __nv_bfloat16* x;  // [T, H] (row stride ldx)
  long ldx;
  const int* ids;          // [T, k] global expert ids (expert g lives on rank g / e_local)
  // symmetric buffers: local views and every rank's address
  const unsigned* flags;                     // this rank's flag array
  unsigned* peer_flags[kEpMaxRanks];
  const int* table;                          // this rank's [W src][W dst][E_l] count table
  int* peer_table[kEpMaxRanks];
  const int* recv_tag;                       // [max_recv][4] (src, token, slot, 0)
  int* peer_recv_tag[kEpMaxRanks];
  __nv_bfloat16* peer_recv_x[kEpMaxRanks];   // [max_recv, H] expert-major rows
  __nv_bfloat16* peer_comb[kEpMaxRanks];     // [T_max, k, H] returned expert outputs
  // expert outputs of the received rows (for the return)
  const __nv_bfloat16* y;
  long ldy;
  // local bookkeeping
  int* recv_counts;   // [E_l]
  int* recv_offsets;  // [E_l + 1]
  int* send_ctr;      // [W * E_l]
  int* epoch_a;
  int* epoch_b;
  int* epoch_c;
  int* ticket_b;
  int* ticket_c;
  int* ok;            // [3] outcome of the count / row / return waits (0 after a timeout)
  int* status;
  unsigned long long limit_ns;
};

void ep_count(const EpArgs& a, cudaStream_t st);
void ep_send(const EpArgs& a, cudaStream_t st);
void ep_wait(const EpArgs& a, int which, cudaStream_t st);  // which: 0 = rows arrived (B), 1 = returns arrived (C)
void ep_return(const EpArgs& a, cudaStream_t st);

}  // namespace bwn
