// The reference engine's device handle (runtime/device/device.h) on the host: test
// infrastructure only. The reference's own device selection (runtime/device/device.cpp)
// queries a real GPU; the checkers that run the reference's model code on the host emulator
// (oracle/hipsim) define its members here instead: no stream, nothing to select.
#pragma once

#include "runtime/device/device.h"

#include <utility>

namespace navi {
Device Device::open() { return Device(); }
Device::~Device() = default;
Device::Device(Device && o) noexcept : info_(std::move(o.info_)), stream_(o.stream_) { o.stream_ = nullptr; }
Device & Device::operator=(Device && o) noexcept {
    info_ = std::move(o.info_);
    stream_ = o.stream_;
    o.stream_ = nullptr;
    return *this;
}
void Device::refresh_memory() {}
} // namespace navi
