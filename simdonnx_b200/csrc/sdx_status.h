// Status codes shared by the C ABI and the device error word. Values mirror include/sdxcuda.h.
#pragma once

#define SDX_OK 0
#define SDX_ERR_INVALID 1        // bad argument / unsupported shape (no work was enqueued)
#define SDX_ERR_CUDA 2           // a CUDA runtime/driver call failed (message in sdx_last_error)
#define SDX_ERR_OOM 3            // device or pinned allocation failed
#define SDX_ERR_TIMEOUT 4        // host watchdog: the stream did not finish before the deadline
#define SDX_ERR_DEVICE 5         // a kernel reported an error through the device error word
#define SDX_ERR_INJECTED 6       // a fault injected by sdx_fault_inject (tests)
#define SDX_ERR_POISONED 7       // the context saw a device error; close and reopen it
#define SDX_ERR_NOT_SUPPORTED 8  // the op/shape has no CUDA kernel (the core never falls back)

// Device error word codes (first error wins; read back with sdx_device_error).
#define SDX_DEV_WAIT_FULL 0x101u       // MMA issuer timed out waiting for a TMA stage
#define SDX_DEV_WAIT_EMPTY 0x102u      // producer timed out waiting for a free stage
#define SDX_DEV_WAIT_ACC_FULL 0x103u   // epilogue timed out waiting for an accumulator
#define SDX_DEV_WAIT_ACC_EMPTY 0x104u  // MMA issuer timed out waiting for the epilogue
#define SDX_DEV_WAIT_DRAIN 0x105u      // wind-down wait for in-flight copies / MMAs timed out
#define SDX_DEV_TEST_WAIT 0x1F0u       // the self-test wait kernel timed out (expected in its test)
#define SDX_DEV_NONFINITE 0x201u       // the fused CTC head saw a non-finite logit (the reference throws)
