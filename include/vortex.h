/*
 * vortex.h — the subset of the Vortex runtime API (runtime/include/vortex.h of
 * the Vortex GPGPU project, located through VORTEX_HOME by akili-bench's
 * config.mk.in:1-17) that akili-bench's kbt_* and flash host harnesses call.
 *
 * libakili_vortex.so implements it on CUDA: buffers are device allocations,
 * `vx_mem_address` returns the CUDA device pointer, `vx_upload_kernel_file`
 * selects which akili_<bench>() entry `vx_start` runs, and `vx_ready_wait`
 * synchronises the stream.  An unchanged benchmarks/<bench>/main.cpp builds
 * against this header and that library and runs on a B200.
 *
 * Signatures follow the call sites, e.g. benchmarks/kbt_sgemm/main.cpp:76-113
 * and benchmarks/flash/main.cpp:172-311.  Every function returns 0 on success.
 */
#ifndef AKILI_VORTEX_H_
#define AKILI_VORTEX_H_

#include <stddef.h>
#include <stdint.h>
#include <stdio.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef void* vx_device_h;
typedef void* vx_buffer_h;

/* capability ids for vx_dev_caps */
#define VX_CAPS_VERSION           0x0
#define VX_CAPS_NUM_THREADS       0x1
#define VX_CAPS_NUM_WARPS         0x2
#define VX_CAPS_NUM_CORES         0x3
#define VX_CAPS_CACHE_LINE_SIZE   0x4
#define VX_CAPS_GLOBAL_MEM_SIZE   0x5
#define VX_CAPS_LOCAL_MEM_SIZE    0x6
#define VX_CAPS_ISA_FLAGS         0x7
#define VX_CAPS_NUM_MEM_BANKS     0x8
#define VX_CAPS_MEM_BANK_SIZE     0x9

/* buffer access flags for vx_mem_alloc */
#define VX_MEM_READ               0x1
#define VX_MEM_WRITE              0x2
#define VX_MEM_READ_WRITE         0x3

/* timeout for vx_ready_wait, in milliseconds */
#define VX_MAX_TIMEOUT            (24ull * 60 * 60 * 1000)

int vx_dev_open(vx_device_h* hdevice);
int vx_dev_close(vx_device_h hdevice);
int vx_dev_caps(vx_device_h hdevice, uint32_t caps_id, uint64_t* value);

int vx_mem_alloc(vx_device_h hdevice, uint64_t size, int flags, vx_buffer_h* hbuffer);
int vx_mem_free(vx_buffer_h hbuffer);
int vx_mem_address(vx_buffer_h hbuffer, uint64_t* address);

int vx_copy_to_dev(vx_buffer_h hbuffer, const void* host_ptr, uint64_t dst_offset, uint64_t size);
int vx_copy_from_dev(void* host_ptr, vx_buffer_h hbuffer, uint64_t src_offset, uint64_t size);

int vx_start(vx_device_h hdevice, vx_buffer_h hkernel, vx_buffer_h harguments);
int vx_ready_wait(vx_device_h hdevice, uint64_t timeout);

int vx_upload_kernel_file(vx_device_h hdevice, const char* filename, vx_buffer_h* hbuffer);
int vx_upload_bytes(vx_device_h hdevice, const void* content, uint64_t size, vx_buffer_h* hbuffer);

int vx_check_occupancy(vx_device_h hdevice, uint32_t group_size, uint32_t* max_localmem);

/* Performance-counter dump (benchmarks/attention/main.cpp:248 calls it after
 * each launch).  The B200 backend has no Vortex counters: it writes nothing
 * and returns 0. */
int vx_dump_perf(vx_device_h hdevice, FILE* stream);

#ifdef __cplusplus
}
#endif
#endif
