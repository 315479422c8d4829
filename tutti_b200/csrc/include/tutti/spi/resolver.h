#pragma once
// Resolver SPI: URI -> immutable ResolvedTarget (logical size, a payload that is
// private between the resolver and the DataPath it recommends, and the key of
// that DataPath). Parity: reference csrc/include/tutti/spi/storage_target_resolver.h:32-124.

#include <cstdint>
#include <memory>
#include <string>
#include <string_view>
#include <utility>

#include <tutti/status.h>

namespace tutti {

struct ResolveOptions {
    std::string scheme;
};

class ResolvedTarget {
public:
    ResolvedTarget() = default;
    ResolvedTarget(ResolvedTarget&&) noexcept = default;
    ResolvedTarget& operator=(ResolvedTarget&&) noexcept = default;
    ResolvedTarget(const ResolvedTarget&) = delete;
    ResolvedTarget& operator=(const ResolvedTarget&) = delete;

    std::string_view resolver_type_id() const noexcept { return s_ ? s_->resolver_type : ""; }
    std::string_view payload_type_id() const noexcept { return s_ ? s_->payload_type : ""; }
    std::uint32_t source_api_version() const noexcept { return s_ ? s_->api_version : 0; }
    std::uint64_t logical_size() const noexcept { return s_ ? s_->logical_size : 0; }
    std::string_view recommended_data_path_key() const noexcept { return s_ ? s_->datapath_key : ""; }
    std::string_view uri() const noexcept { return s_ ? s_->uri : ""; }
    bool valid() const noexcept { return s_ != nullptr; }

    // Typed view of the payload; fails closed on a type or version mismatch.
    template <typename Payload>
    Result<const Payload*> view(std::string_view payload_type, std::uint32_t api_version) const {
        if (!s_) return Result<const Payload*>::Failure({StatusCode::UNSUPPORTED, "empty target"});
        if (s_->payload_type != payload_type)
            return Result<const Payload*>::Failure(
                {StatusCode::UNSUPPORTED, "payload type mismatch: have " + s_->payload_type});
        if (s_->api_version != api_version)
            return Result<const Payload*>::Failure({StatusCode::UNSUPPORTED, "payload API version mismatch"});
        return static_cast<const Payload*>(s_->payload.get());
    }

    template <typename Payload>
    static ResolvedTarget make(std::string resolver_type, std::string payload_type,
                               std::uint32_t api_version, std::uint64_t logical_size,
                               std::string datapath_key, std::string uri,
                               std::shared_ptr<const Payload> payload) {
        ResolvedTarget t;
        t.s_ = std::make_shared<Storage>();
        t.s_->resolver_type = std::move(resolver_type);
        t.s_->payload_type = std::move(payload_type);
        t.s_->api_version = api_version;
        t.s_->logical_size = logical_size;
        t.s_->datapath_key = std::move(datapath_key);
        t.s_->uri = std::move(uri);
        t.s_->payload = std::static_pointer_cast<const void>(payload);
        return t;
    }

private:
    struct Storage {
        std::string resolver_type, payload_type, datapath_key, uri;
        std::uint32_t api_version = 0;
        std::uint64_t logical_size = 0;
        std::shared_ptr<const void> payload;
    };
    std::shared_ptr<Storage> s_;
};

class StorageTargetResolver {
public:
    virtual ~StorageTargetResolver() = default;
    virtual Result<ResolvedTarget> resolve(std::string_view uri, const ResolveOptions& options) = 0;
};

}  // namespace tutti
