#pragma once
/* Allocation-free entry point of the GPU NVMe io path.
 *
 * This entry point has no counterpart in the reference. It exists for callers
 * that cannot allocate GPU memory at the moment they move KV: serving engines
 * that hand every free byte of HBM to their KV pool at start-up, so that a
 * later cudaMalloc in the middle of a step can fail with out-of-memory, and
 * embedders that reach this library through a plain C ABI (a C, C++ or Rust
 * serving process) and own no CUDA allocator of their own to lend it. The call
 * copies the caller's command list into a fixed device array that is part of
 * the library image and launches the same fused io kernel the runtime uses.
 *
 * The call is synchronous: it enqueues its copies and the kernel on the
 * caller's stream, waits for that stream, reads the per-command status words
 * on the host and only then returns.
 *
 * Limits (per call): at most TUTTI_NOALLOC_MAX_COMMANDS commands and
 * TUTTI_NOALLOC_MAX_PIECES pieces; larger batches are refused with
 * TUTTI_NOALLOC_E_TOO_LARGE before anything is launched. The fixed array is
 * about 2.3 MiB and every GPU that loads the library holds it until the
 * process exits.
 *
 * Sharing: every call on a device uses the same array, which keeps the
 * previous call's contents (the work cursor and the status words are cleared
 * by each call before its launch). Calls that overlap on the GPU, from two
 * threads or on two streams, race on that array; serialise them.
 *
 * Set-up: the first call on a device, with that device current, looks up the
 * array's device address (cudaGetSymbolAddress) once; make that first call
 * before any stream capture begins.
 */

#include <stdint.h>

#include <cuda_runtime_api.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TUTTI_NOALLOC_API __attribute__((visibility("default")))

#define TUTTI_NOALLOC_MAX_COMMANDS 4096u
#define TUTTI_NOALLOC_MAX_PIECES 131072u
#define TUTTI_NOALLOC_MAX_LEASES 256u

/* One command: a contiguous logical range of one opened target (target_row =
 * the DataPath target token), read or written through one staging slot. The
 * fields sit at the io kernel's own command offsets (checked at compile time),
 * so the list is copied to the device as is.
 *   opcode:    2 = read (restore), 1 = write (store);
 *   transform: must be 0 (stored bytes equal memory bytes);
 *   replicas:  must be 0 or 1 (the command's bytes go to one destination). */
typedef struct {
    uint64_t logical;
    uint32_t target_row;
    uint32_t bytes;
    uint32_t first_piece;
    uint32_t n_pieces;
    uint16_t opcode;
    uint16_t transform;
    uint32_t replicas;
} tutti_noalloc_command;

/* Where bytes [off, off + bytes) of a command live in caller memory
 * (a device address, 16-byte aligned). */
typedef struct {
    uint64_t mem;
    uint32_t off;
    uint32_t bytes;
} tutti_noalloc_piece;

#define TUTTI_NOALLOC_OK 0
#define TUTTI_NOALLOC_E_ARGS -1
#define TUTTI_NOALLOC_E_TOO_LARGE -2
#define TUTTI_NOALLOC_E_BUSY -3
#define TUTTI_NOALLOC_E_CUDA -4
#define TUTTI_NOALLOC_E_SETUP -5

/* Runs `n_commands` commands through the GpuNvmeDataPath at `data_path`
 * (obtained from a runtime built earlier) on `stream` and waits for them.
 * `cmd_status` (host, n_commands words) receives 0 per successful command,
 * else the io kernel's status word (0xFFFFFFFF: the command never ran).
 * Returns TUTTI_NOALLOC_OK, the number of failed commands (> 0), or a
 * negative TUTTI_NOALLOC_E_* code; tutti_noalloc_last_error() describes it. */
TUTTI_NOALLOC_API int tutti_nvme_io_noalloc(void* data_path, const tutti_noalloc_command* commands, uint32_t n_commands,
                          const tutti_noalloc_piece* pieces, uint32_t n_pieces, uint32_t* cmd_status,
                          cudaStream_t stream);

TUTTI_NOALLOC_API const char* tutti_noalloc_last_error(void);

#ifdef __cplusplus
}
#endif
