// A value looked up per CUDA context and kept while that context stays
// current: the device address of a `__device__` array, which is valid only
// in the context whose module load placed it.  A device reset or a context
// the caller creates loads the module again at another address, so the
// value is looked up again whenever the current context is not the one it
// was taken in.  Contexts are told apart by their process-unique id
// (cuCtxGetId), not by their handle, which a new context can reuse.
//
// Host-only C++ with no CUDA dependency, so that its logic can be checked on
// a machine without a GPU.
#pragma once

#include <cstdint>
#include <mutex>

namespace mhcp {

template <int kSlots>
class ContextCache {
public:
    // The value for context `ctx_id` in slot `slot` (the device number):
    // the kept one when it was taken in that context, else lookup(&value),
    // kept on success.  ctx_id 0 means "context unknown": the value is looked
    // up on every call and not kept.  Returns lookup's status, or the
    // kept value's 0.
    template <class Lookup>
    int get(int slot, unsigned long long ctx_id, Lookup lookup, void** value)
    {
        if (slot < 0 || slot >= kSlots) return lookup(value);
        std::lock_guard<std::mutex> hold(mu_);
        Entry& e = entries_[slot];
        if (ctx_id != 0 && e.ctx_id == ctx_id) {
            *value = e.value;
            return 0;
        }
        void* v = nullptr;
        const int status = lookup(&v);
        if (status != 0) return status;
        e.ctx_id = ctx_id;  // 0 never matches, so an unknown context looks up again
        e.value = v;
        *value = v;
        return 0;
    }

    // Whether slot `slot` holds a value taken in context `ctx_id`.
    bool holds(int slot, unsigned long long ctx_id)
    {
        if (slot < 0 || slot >= kSlots || ctx_id == 0) return false;
        std::lock_guard<std::mutex> hold(mu_);
        return entries_[slot].ctx_id == ctx_id;
    }

private:
    struct Entry {
        unsigned long long ctx_id = 0;
        void* value = nullptr;
    };
    std::mutex mu_;
    Entry entries_[kSlots];
};

}  // namespace mhcp
