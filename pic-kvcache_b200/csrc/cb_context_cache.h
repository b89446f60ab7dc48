// Host-side table from a CUDA context handle to a value recorded in that
// context (here: the device address of a file-scope __device__ array).  Plain
// C++ with opaque keys, so its behaviour is checked on a machine without a GPU.
// Not thread-safe by itself: callers hold their own mutex.
#pragma once

#include <stddef.h>

namespace cb {

template <typename Value, int Slots>
class ContextTable {
 public:
  // Value recorded for `context`, or `missing` if none.
  Value find(const void* context, Value missing) const {
    for (int i = 0; i < used_; ++i)
      if (keys_[i] == context) return values_[i];
    return missing;
  }

  // Records `value` for `context`, replacing an earlier value for the same
  // handle (a context destroyed and created again may reuse its handle, and
  // its symbols may then live elsewhere).  Returns false when the table is full.
  bool store(const void* context, Value value) {
    for (int i = 0; i < used_; ++i)
      if (keys_[i] == context) {
        values_[i] = value;
        return true;
      }
    if (used_ == Slots) return false;
    keys_[used_] = context;
    values_[used_] = value;
    ++used_;
    return true;
  }

  int size() const { return used_; }

 private:
  const void* keys_[Slots] = {};
  Value values_[Slots] = {};
  int used_ = 0;
};

}  // namespace cb
