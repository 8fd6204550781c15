/*
 * gnn_b200_umprof.h — C ABI of libgnnb200_umprof.so: unified-memory migration
 * counters collected in-process through CUPTI, without nsys.
 *
 * Replaces the measurement half of the reference's run/profile_spmm_migration.py
 * (nsys profile + SQLite export + the queries of :303-461): host-to-device and
 * device-to-host migration bytes and GPU page faults over the feature matrix's
 * address range, reported as HtoD_bytes / DtoH_bytes / GPU_faults (:571-575).
 * Kept apart from libgnnb200.so so that the aggregation library never links
 * CUPTI. Status codes are gnn_status values (gnn_b200.h).
 */
#ifndef GNN_B200_UMPROF_H_
#define GNN_B200_UMPROF_H_

#include <stdint.h>

#include "gnn_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

typedef struct gnn_um_totals {
  double htod_bytes;        /* unified-memory bytes migrated host -> device       */
  double dtoh_bytes;        /* unified-memory bytes migrated device -> host       */
  double gpu_page_faults;   /* GPU page faults (page-fault groups per page)       */
  double cpu_page_faults;   /* CPU page-fault records                              */
  double thrashing_bytes;   /* bytes of regions the driver saw thrashing          */
  double throttling_events; /* throttling operations                               */
  double remote_map_bytes;  /* bytes remote-mapped instead of migrated            */
  uint64_t records;         /* records that passed the filters                    */
  uint64_t dropped_records; /* records CUPTI dropped (buffers full), all time      */
} gnn_um_totals;

/* Enables collection of CUPTI unified-memory counter records for this process.
 * Call it before the first CUDA call of the process where possible (CUPTI may
 * refuse or miss records for contexts created earlier). */
int gnn_um_profiler_start(void);
/* Hands every buffered record to the library (cuptiActivityFlushAll). */
int gnn_um_profiler_flush(void);
/* Flushes and disables collection; the stored records stay readable. */
int gnn_um_profiler_stop(void);
/* Drops the stored records. */
int gnn_um_profiler_clear(void);
/* CUPTI timestamp in ns (the clock of the records), 0 on failure. */
uint64_t gnn_um_profiler_timestamp(void);
/* Sums the stored records: migrations whose [address, address + bytes)
 * overlaps [range_begin, range_end) and faults whose address lies in it
 * (range 0, 0 = every address), and whose [start, end) overlaps
 * [t_begin, t_end) (0, 0 = all time). Call gnn_um_profiler_flush first. */
int gnn_um_profiler_totals(uint64_t range_begin, uint64_t range_end, uint64_t t_begin, uint64_t t_end,
                           gnn_um_totals* out);
/* Number of counter kinds collection runs with, as a prefix of: HtoD bytes,
 * DtoH bytes, GPU page faults, CPU page faults, thrashing, throttling, remote
 * maps (platforms lacking a kind run with fewer; at least the first two). */
int gnn_um_profiler_enabled_kinds(void);
const char* gnn_um_profiler_last_error(void);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* GNN_B200_UMPROF_H_ */
