/* ridgefill_team.h -- tensor parallelism over one prompt: one process per GPU, each rank's buffers mapped into its
 * peers' address spaces, and the NVLink kernels that gather a column-split matrix and order the ranks.
 *
 * No counterpart in the reference: its engine replicates the projector on every tensor-parallel rank and reduces
 * with its own all-reduce (notes/tp-map.md:28-29,48-49); the value heads' spans are its (tests/kernel_test.cpp:
 * 1458-1577). Here the projector's output columns are split across ranks and reassembled by
 * ridgefill_gather_columns, so each rank computes 1/world of every projector.
 *
 * The protocol. Every rank holds a counter array (unsigned 64-bit, device memory, zeroed once) and maps every
 * peer's; counters only grow. A rank's gather of slot s adds ridgefill_team_gather_ctas() arrivals to slot s of
 * every peer once its stores are visible there; after its e-th pass each rank's slot s has received
 * e * (world - 1) * ridgefill_team_gather_ctas() arrivals, which ridgefill_team_wait waits for before the data is
 * read. ridgefill_team_barrier adds one arrival to every peer's slot and waits for e * (world - 1). Every wait gives
 * up after 2 s (ridgefill_device_error then reports 0x301) and the stream continues: a dead peer costs an error,
 * never a hang. Nothing here allocates; no multicast of any kind is used.
 */
#ifndef RIDGEFILL_TEAM_H
#define RIDGEFILL_TEAM_H

#include <stdint.h>

#include "rad_abi.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Arrivals one gather adds to a peer's counter slot (its CTAs). */
int ridgefill_team_gather_ctas(void);

/* Export device pointer `ptr` for a peer process: the 64-byte IPC handle of the allocation holding it into
 * `handle`, and its byte offset inside that allocation into *offset. */
int ridgefill_peer_export(const void* ptr, void* handle, int64_t* offset);

/* Map a peer's exported pointer into this process (the current device): *ptr = its address here. */
int ridgefill_peer_import(const void* handle, int64_t offset, void** ptr);

/* Unmap a pointer ridgefill_peer_import returned (with the same offset). */
int ridgefill_peer_release(void* ptr, int64_t offset);

/* On stream `s`: the block of columns [c0, c1) of rows [0, rows) of this rank's bf16 matrix `src` (row pitch `ld`
 * elements) stored into every peer's copy dst[p] (p != rank; the same layout), then the arrivals on slot `slot` of
 * every peer's counters flags[p]. Addresses, the pitch and both column bounds in bytes must be multiples of 16;
 * world <= 8. */
int ridgefill_gather_columns(const uint16_t* src, uint16_t* const* dst, unsigned long long* const* flags, int rank,
                             int world, int64_t rows, int64_t ld, int64_t c0, int64_t c1, int slot, RadStream s);

/* On stream `s`: wait until this rank's counter `slot` (own, device memory) holds at least `expected`. */
int ridgefill_team_wait(const unsigned long long* own, int slot, unsigned long long expected, RadStream s);

/* On stream `s`: an arrival on slot `slot` of every peer's counters, then the wait until flags[rank][slot] holds at
 * least `expected`. */
int ridgefill_team_barrier(unsigned long long* const* flags, int rank, int world, int slot, unsigned long long expected,
                           RadStream s);

#ifdef __cplusplus
}
#endif

#endif /* RIDGEFILL_TEAM_H */
