// C++ entry point of the MPI subset for programs that already hold the job's
// c10d store (the native benchmark tools): the subset starts on that store
// instead of connecting to MASTER_ADDR / MASTER_PORT itself. Everything else
// is as after MPI_Init_thread; MPI_Finalize ends it.
#pragma once

#include <torch/csrc/distributed/c10d/Store.hpp>

namespace mgfa::mpi_shim {

// Collective over all `world` ranks (maps the shared-memory mailbox). Throws
// std::runtime_error on failure; a second call is a no-op. timeout_s > 0 bounds
// every wait of the subset (otherwise MPI_SHIM_TIMEOUT_S, default 600 s).
void init_with_store(c10::intrusive_ptr<c10d::Store> store, int rank, int world,
                     int timeout_s = 0);

}  // namespace mgfa::mpi_shim
