/* Declarations-only stand-in for the few OpenCL types, constants and calls
 * that the reference's include/infvino/ClRuntime.hpp names, so that its
 * Device.hpp (infvino::DeviceInfo) compiles in the C++ boundary test without
 * an OpenCL SDK.  TEST INFRASTRUCTURE ONLY: nothing here is defined or called;
 * the test program never instantiates the OpenCL runtime. */
#ifndef IVB_TEST_CL_STUB_H_
#define IVB_TEST_CL_STUB_H_
#include <stddef.h>
#include <stdint.h>
typedef int32_t cl_int;
typedef uint32_t cl_uint;
typedef uint64_t cl_ulong;
typedef cl_ulong cl_mem_flags;
typedef cl_uint cl_version;
typedef cl_uint cl_buffer_create_type;
typedef struct _cl_platform_id *cl_platform_id;
typedef struct _cl_device_id *cl_device_id;
typedef struct _cl_context *cl_context;
typedef struct _cl_command_queue *cl_command_queue;
typedef struct _cl_mem *cl_mem;
typedef struct _cl_program *cl_program;
typedef struct _cl_kernel *cl_kernel;
typedef struct _cl_event *cl_event;
typedef struct {
  size_t origin;
  size_t size;
} cl_buffer_region;
#define CL_SUCCESS 0
#define CL_MEM_READ_WRITE ((cl_mem_flags)1)
#define CL_BUFFER_CREATE_TYPE_REGION 0x1220
#ifdef __cplusplus
extern "C" {
#endif
cl_int clReleaseMemObject(cl_mem);
cl_mem clCreateSubBuffer(cl_mem, cl_mem_flags, cl_buffer_create_type, const void *, cl_int *);
#ifdef __cplusplus
}
#endif
#endif
