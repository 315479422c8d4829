#pragma once
// RAII: make `accel_id` the current CUDA device for a scope and restore the
// caller's device afterwards (reference accelerator_device_guard.h:89).

#include <cuda_runtime_api.h>

#include <tutti/status.h>

namespace tutti {

class DeviceGuard {
public:
    explicit DeviceGuard(int accel_id) {
        if (accel_id < 0) return;
        if (cudaGetDevice(&prev_) != cudaSuccess) {
            cudaGetLastError();
            prev_ = -1;
        }
        if (prev_ != accel_id) {
            cudaError_t e = cudaSetDevice(accel_id);
            if (e != cudaSuccess) {
                cudaGetLastError();
                status_ = Status(StatusCode::DEVICE_ERROR,
                                 std::string("cudaSetDevice: ") + cudaGetErrorString(e));
            } else {
                restore_ = prev_ >= 0;
            }
        }
    }
    ~DeviceGuard() {
        if (restore_) cudaSetDevice(prev_);
    }
    DeviceGuard(const DeviceGuard&) = delete;
    DeviceGuard& operator=(const DeviceGuard&) = delete;
    const Status& status() const { return status_; }

private:
    int prev_ = -1;
    bool restore_ = false;
    Status status_;
};

}  // namespace tutti
