#pragma once
namespace maloq {
// Read (and optionally clear) the device error word: 0 = none, codes in common.cuh, -1 = read failed.
int error_status(bool clear);
// True when the library was compiled with MALOQ_BOUNDS_CHECK (device index checks).
bool bounds_checked();
}  // namespace maloq
