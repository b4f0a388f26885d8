// Device-side signalling between GPUs that mapped each other's memory (CUDA IPC): release/acquire flag words at
// system scope, L1-bypassing vector loads of peer-written data, and bounded flag waits (globaltimer deadline; a
// time-out records ERR_PEER_TIMEOUT in the error word instead of spinning forever).
#pragma once
#include "common.cuh"

namespace tgo {

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ void flag_store_release(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t flag_load_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
// 16-byte load that bypasses L1 (data written by another GPU after a flag handshake)
__device__ __forceinline__ uint4 ld_v4_volatile(const void* ptr) {
  uint4 u;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
               : "l"(ptr)
               : "memory");
  return u;
}
__device__ __forceinline__ __nv_bfloat16 ld_bf16_volatile(const __nv_bfloat16* ptr) {
  unsigned short u;
  asm volatile("ld.volatile.global.u16 %0, [%1];" : "=h"(u) : "l"(ptr) : "memory");
  return __ushort_as_bfloat16(u);
}
// Wait until *p == v (epochs only grow; equality of the 32-bit value is what is compared). Bounded.
__device__ __forceinline__ bool flag_wait(const uint32_t* p, uint32_t v, uint64_t deadline_ns, int* err) {
  while (flag_load_acquire(p) != v) {
    if (global_ns() > deadline_ns) {
      record_error(err, ERR_PEER_TIMEOUT);
      return false;
    }
  }
  return true;
}

}  // namespace tgo
