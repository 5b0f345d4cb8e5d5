// Checks the per-context cache of the no-allocation backward's array
// address (mhc-proj_b200/csrc/context_cache.h) with a fake lookup: no GPU.
// Prints "ok" and exits 0 when every check holds.
#include <cstdio>

#include "context_cache.h"

static int lookups = 0;
static void* next_address = nullptr;

static int fake_lookup(void** v)
{
    ++lookups;
    *v = next_address;
    return 0;
}

static int fail = 0;
#define CHECK(c)                                            \
    do {                                                    \
        if (!(c)) {                                         \
            std::printf("failed: %s (line %d)\n", #c, __LINE__); \
            fail = 1;                                       \
        }                                                   \
    } while (0)

int main()
{
    mhcp::ContextCache<4> cache;
    void* got = nullptr;
    char a, b, c;

    // first call in context 7 on device 0 looks up; later calls do not
    next_address = &a;
    CHECK(cache.get(0, 7, fake_lookup, &got) == 0 && got == &a && lookups == 1);
    next_address = &b;
    CHECK(cache.get(0, 7, fake_lookup, &got) == 0 && got == &a && lookups == 1);
    CHECK(cache.holds(0, 7) && !cache.holds(0, 8) && !cache.holds(1, 7));

    // a new context on the same device (a reset, or a context the caller
    // made) has a new id: looked up again, and the new address kept
    CHECK(cache.get(0, 8, fake_lookup, &got) == 0 && got == &b && lookups == 2);
    CHECK(cache.get(0, 8, fake_lookup, &got) == 0 && got == &b && lookups == 2);

    // going back to the first context looks up again (its module may have
    // been loaded anew)
    next_address = &c;
    CHECK(cache.get(0, 7, fake_lookup, &got) == 0 && got == &c && lookups == 3);

    // devices are kept apart
    next_address = &a;
    CHECK(cache.get(1, 7, fake_lookup, &got) == 0 && got == &a && lookups == 4);
    CHECK(cache.get(0, 7, fake_lookup, &got) == 0 && got == &c && lookups == 4);

    // an unknown context (id 0) is never kept: looked up on every call
    CHECK(cache.get(2, 0, fake_lookup, &got) == 0 && lookups == 5);
    CHECK(cache.get(2, 0, fake_lookup, &got) == 0 && lookups == 6);
    CHECK(!cache.holds(2, 0));

    // a failed lookup is returned and nothing is kept
    auto failing = [](void** v) -> int { *v = nullptr; return 42; };
    CHECK(cache.get(3, 9, failing, &got) == 42);
    CHECK(!cache.holds(3, 9));
    next_address = &b;
    CHECK(cache.get(3, 9, fake_lookup, &got) == 0 && got == &b && lookups == 7);

    // a device number outside the table is served without keeping anything
    CHECK(cache.get(17, 5, fake_lookup, &got) == 0 && lookups == 8);
    CHECK(cache.get(17, 5, fake_lookup, &got) == 0 && lookups == 9);

    if (!fail) std::printf("ok\n");
    return fail;
}
