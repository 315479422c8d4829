#pragma once
// Status / Result<T>: the error vocabulary of every public and SPI call.
//
// Parity: the code set and the "Result never holds OK without a value" rule
// follow the reference's public status header (csrc/include/tutti/status.h:21-130).

#include <optional>
#include <string>
#include <utility>

namespace tutti {

enum class StatusCode {
    OK,
    INVALID_ARGUMENT,
    OUT_OF_RANGE,
    NOT_FOUND,
    UNSUPPORTED,
    NOT_READY,
    BUSY,
    RESOURCE_EXHAUSTED,
    TIMEOUT,
    DEVICE_ERROR,
    DATA_LOSS,
    INTERNAL,
    PERMISSION_DENIED,
};

inline const char* status_code_name(StatusCode c) noexcept {
    switch (c) {
        case StatusCode::OK: return "OK";
        case StatusCode::INVALID_ARGUMENT: return "INVALID_ARGUMENT";
        case StatusCode::OUT_OF_RANGE: return "OUT_OF_RANGE";
        case StatusCode::NOT_FOUND: return "NOT_FOUND";
        case StatusCode::UNSUPPORTED: return "UNSUPPORTED";
        case StatusCode::NOT_READY: return "NOT_READY";
        case StatusCode::BUSY: return "BUSY";
        case StatusCode::RESOURCE_EXHAUSTED: return "RESOURCE_EXHAUSTED";
        case StatusCode::TIMEOUT: return "TIMEOUT";
        case StatusCode::DEVICE_ERROR: return "DEVICE_ERROR";
        case StatusCode::DATA_LOSS: return "DATA_LOSS";
        case StatusCode::INTERNAL: return "INTERNAL";
        case StatusCode::PERMISSION_DENIED: return "PERMISSION_DENIED";
    }
    return "?";
}

class Status {
public:
    Status() = default;
    Status(StatusCode code, std::string message)
        : code_(code), message_(std::move(message)) {}
    static Status Ok() { return Status(); }

    bool ok() const noexcept { return code_ == StatusCode::OK; }
    StatusCode code() const noexcept { return code_; }
    const std::string& message() const noexcept { return message_; }
    std::string to_string() const {
        return ok() ? std::string("OK")
                    : std::string(status_code_name(code_)) + ": " + message_;
    }

private:
    StatusCode code_ = StatusCode::OK;
    std::string message_;
};

template <typename T>
class Result {
public:
    Result(T value) : value_(std::move(value)) {}  // NOLINT: implicit success
    explicit Result(Status status) : status_(std::move(status)) {
        if (status_.ok())
            status_ = Status(StatusCode::INTERNAL,
                             "Result built from OK status without a value");
    }
    static Result Success(T value) { return Result(std::move(value)); }
    static Result Failure(Status status) { return Result(std::move(status)); }

    bool ok() const noexcept { return status_.ok(); }
    bool has_value() const noexcept { return value_.has_value(); }
    const Status& status() const noexcept { return status_; }
    T& value() & { return *value_; }
    const T& value() const& { return *value_; }
    T&& value() && { return std::move(*value_); }

private:
    std::optional<T> value_;
    Status status_;
};

#define TUTTI_RETURN_IF_ERROR(expr)            \
    do {                                       \
        ::tutti::Status _st = (expr);          \
        if (!_st.ok()) return _st;             \
    } while (0)

#define TUTTI_RETURN_IF_ERROR_R(R, expr)           \
    do {                                           \
        ::tutti::Status _st = (expr);              \
        if (!_st.ok()) return R::Failure(_st);     \
    } while (0)

}  // namespace tutti
