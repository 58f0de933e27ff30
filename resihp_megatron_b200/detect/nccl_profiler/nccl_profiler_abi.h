// Declarations of NCCL's profiler-plugin interface, version 5 (NCCL >= 2.26 loads the exported
// symbol `ncclProfiler_v5`).  Only the types this plugin touches are declared; the member order
// and widths of every struct follow the published v5 ABI exactly, since NCCL passes these
// structures by pointer.
#pragma once

#include <cstddef>
#include <cstdint>
#include <sys/types.h>

extern "C" {

typedef enum {
  ncclSuccess = 0,
  ncclUnhandledCudaError = 1,
  ncclSystemError = 2,
  ncclInternalError = 3,
  ncclInvalidArgument = 4,
  ncclInvalidUsage = 5,
  ncclRemoteError = 6
} ncclResult_t;

// The logger is never called here; only its pointer width matters.
typedef void (*ncclDebugLogger_t)(int level, unsigned long flags, const char* file, int line, const char* fmt, ...);

enum {
  ncclProfileGroup = 1 << 0,
  ncclProfileColl = 1 << 1,
  ncclProfileP2p = 1 << 2,
  ncclProfileProxyOp = 1 << 3,
  ncclProfileProxyStep = 1 << 4,
  ncclProfileProxyCtrl = 1 << 5,
  ncclProfileKernelCh = 1 << 6,
  ncclProfileNetPlugin = 1 << 7,
  ncclProfileGroupApi = 1 << 8,
  ncclProfileCollApi = 1 << 9,
  ncclProfileP2pApi = 1 << 10,
  ncclProfileKernelLaunch = 1 << 11,
};

typedef int ncclProfilerEventState_v5_t;

typedef struct {
  uint64_t type;
  void* parentObj;
  int rank;
  union {
    struct {
      bool graphCaptured;
      int groupDepth;
    } groupApi;
    struct {
      const char* func;
      size_t count;
      const char* datatype;
      int root;
      void* stream;
      bool graphCaptured;
    } collApi;
    struct {
      const char* func;
      size_t count;
      const char* datatype;
      void* stream;
      bool graphCaptured;
    } p2pApi;
    struct {
      void* stream;
    } kernelLaunch;
    struct {
      uint64_t seqNumber;
      const char* func;
      void const* sendBuff;
      void* recvBuff;
      size_t count;
      int root;
      const char* datatype;
      uint8_t nChannels;
      uint8_t nWarps;
      const char* algo;
      const char* proto;
      void* parentGroup;
    } coll;
    struct {
      const char* func;
      void* buff;
      const char* datatype;
      size_t count;
      int peer;
      uint8_t nChannels;
      void* parentGroup;
    } p2p;
    struct {
      pid_t pid;
      uint8_t channelId;
      int peer;
      int nSteps;
      int chunkSize;
      int isSend;
    } proxyOp;
    struct {
      int step;
    } proxyStep;
    struct {
      uint8_t channelId;
      uint64_t pTimer;
    } kernelCh;
    struct {
      int64_t id;
      void* data;
    } netPlugin;
  };
} ncclProfilerEventDescr_v5_t;

typedef union {
  struct {
    size_t transSize;
  } proxyStep;
  struct {
    int appendedProxyOps;
  } proxyCtrl;
  struct {
    void* data;
  } netPlugin;
  struct {
    uint64_t pTimer;
  } kernelCh;
} ncclProfilerEventStateArgs_v5_t;

typedef struct {
  const char* name;
  ncclResult_t (*init)(void** context, uint64_t commId, int* eActivationMask, const char* commName, int nNodes,
                       int nranks, int rank, ncclDebugLogger_t logfn);
  ncclResult_t (*startEvent)(void* context, void** eHandle, ncclProfilerEventDescr_v5_t* eDescr);
  ncclResult_t (*stopEvent)(void* eHandle);
  ncclResult_t (*recordEventState)(void* eHandle, ncclProfilerEventState_v5_t eState,
                                   ncclProfilerEventStateArgs_v5_t* eStateArgs);
  ncclResult_t (*finalize)(void* context);
} ncclProfiler_v5_t;

}  // extern "C"
