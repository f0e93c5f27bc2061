// ref_hooks.cpp -- global operator new/delete that copy out the fifth buffer
// allocated after ref_capture_arm(): inside the reference's verify_attn that
// is hORef, its CPU output (allocation order hQ, hK, hV, hO, hORef,
// tuning/utils.cuh:89-90).  TEST INFRASTRUCTURE ONLY (part of oracle/_ref).
#include <cstdlib>
#include <cstring>
#include <new>
#include <vector>

static thread_local int tl_armed = 0;
static thread_local int tl_index = 0;
static thread_local void* tl_target = nullptr;
static thread_local size_t tl_bytes = 0;
static thread_local unsigned char* tl_saved = nullptr;
static thread_local int tl_have = 0;

extern "C" void ref_capture_arm(size_t oref_bytes) {
  std::free(tl_saved);
  tl_saved = static_cast<unsigned char*>(std::malloc(oref_bytes ? oref_bytes : 1));
  tl_bytes = oref_bytes;
  tl_index = 0;
  tl_target = nullptr;
  tl_have = 0;
  tl_armed = 1;
}

extern "C" int ref_capture_take(void* out, size_t nbytes) {
  tl_armed = 0;
  if (!tl_have || nbytes != tl_bytes) return 1;
  std::memcpy(out, tl_saved, nbytes);
  return 0;
}

void* operator new(size_t n) {
  void* p = std::malloc(n ? n : 1);
  if (!p) throw std::bad_alloc();
  if (tl_armed && ++tl_index == 5) tl_target = p;
  return p;
}

void operator delete(void* p) noexcept {
  if (tl_armed && p != nullptr && p == tl_target && tl_saved != nullptr) {
    std::memcpy(tl_saved, p, tl_bytes);
    tl_have = 1;
    tl_target = nullptr;
  }
  std::free(p);
}

void operator delete(void* p, size_t) noexcept { operator delete(p); }
