#pragma once
namespace maloq {
// Read (and optionally clear) the device error word: 0 = none, codes in common.cuh, -1 = read failed.
int error_status(bool clear);
}  // namespace maloq
