// b2g_internal.h — helpers shared between the library's translation units
// (not part of the C ABI; hidden symbols).
#pragma once

namespace b2g {

// Device address of the current device's error word (the one
// b2g_read_device_error reports), created on first use; nullptr when no
// sm_100 device is current.
int* current_error_word();

// Bound on every device-side wait, in ns (B2G_WAIT_LIMIT_MS, default 2 s).
long long current_wait_limit_ns();

// Launch with programmatic stream serialization (0 when built without it).
bool pdl_enabled();

}  // namespace b2g
