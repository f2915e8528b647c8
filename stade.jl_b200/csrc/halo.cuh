// Communicator services used by the sweeps themselves (slab halo exchange,
// a small sum across ranks); implemented in ddp.cu next to stade_comm.
#pragma once

#include "common.cuh"

namespace stade {

// Sends this slab's first and last rows to the neighbouring slabs (rank - 1
// and rank + 1, periodic) and receives their edge rows into top_halo /
// bottom_halo, on a side stream ordered after the work queued on `s` so far;
// `s` itself is not held up. comm == nullptr or one rank: the slab is the
// whole grid and its halos are copies of its own edge rows, on `s`.
stade_status halo_begin(stade_comm* c, const double* first_row, const double* last_row,
                        double* top_halo, double* bottom_halo, int64_t count, cudaStream_t s);
// Makes `s` wait for the exchange halo_begin queued.
stade_status halo_end(stade_comm* c, cudaStream_t s);
// In-place sum of `count` doubles across ranks on `s` (no-op for one rank).
stade_status comm_allreduce_f64(stade_comm* c, double* buf, int64_t count, cudaStream_t s);
// Waits for `s` to drain, bounded by the communicator's timeout.
stade_status comm_wait_stream(stade_comm* c, cudaStream_t s);
int comm_size(const stade_comm* c);

}  // namespace stade
