#pragma once

/// @file common.hpp
/// @brief Result<T, E> error type, thread-safe logger and check macros.
///
/// Same public surface as the reference's core utilities
/// (include/tensorbit/core/common.hpp:89-417): `Unexpected<E>` /
/// `unexpected(e)`, `Result<T, E>` and `Result<void, E>`, the `Logger`
/// singleton with the `TENSORBIT_LOG_*` macros, and `TENSORBIT_CHECK`.
/// Device work goes through the C ABI (tb_kernels.h), whose calls return
/// status codes instead of aborting.

#include <chrono>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <ctime>
#include <format>
#include <mutex>
#include <new>
#include <source_location>
#include <string>
#include <string_view>
#include <type_traits>
#include <utility>

/// Aborts with file/line and message when `cond` is false (common.hpp:89-99).
#define TENSORBIT_CHECK(cond, msg)                                                            \
    do {                                                                                      \
        if (!(cond)) {                                                                        \
            std::fprintf(stderr, "[TENSORBIT ERROR] %s:%d: %s (check `%s` failed)\n",        \
                         std::source_location::current().file_name(),                       \
                         static_cast<int>(std::source_location::current().line()), (msg), #cond); \
            std::abort();                                                                     \
        }                                                                                     \
    } while (0)

namespace tensorbit::core {

// ---------------------------------------------------------------------------
// Logging
// ---------------------------------------------------------------------------

enum class LogLevel : uint8_t { kTrace = 0, kDebug = 1, kInfo = 2, kWarn = 3, kError = 4, kFatal = 5 };

[[nodiscard]] constexpr std::string_view to_string(LogLevel level) noexcept {
    switch (level) {
    case LogLevel::kTrace: return "TRACE";
    case LogLevel::kDebug: return "DEBUG";
    case LogLevel::kInfo: return "INFO";
    case LogLevel::kWarn: return "WARN";
    case LogLevel::kError: return "ERROR";
    case LogLevel::kFatal: return "FATAL";
    }
    return "UNKNOWN";
}

/// Process-wide logger: one line per message on stderr with wall-clock time,
/// level and source location; a mutex keeps lines whole across threads.
class Logger {
public:
    static Logger& instance() {
        static Logger logger;
        return logger;
    }

    void set_level(LogLevel level) noexcept { level_ = level; }
    [[nodiscard]] LogLevel level() const noexcept { return level_; }

    void log(LogLevel level, std::string_view msg,
             const std::source_location& loc = std::source_location::current()) {
        if (level < level_) return;
        const auto now = std::chrono::system_clock::now();
        const auto t = std::chrono::system_clock::to_time_t(now);
        const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(now.time_since_epoch()).count() % 1000;
        std::tm tm{};
        localtime_r(&t, &tm);
        char stamp[32];
        std::strftime(stamp, sizeof(stamp), "%Y-%m-%d %H:%M:%S", &tm);
        std::lock_guard<std::mutex> lk(mu_);
        std::fprintf(stderr, "[%s.%03d] [%.*s] %.*s  (%s:%u)\n", stamp, static_cast<int>(ms),
                     static_cast<int>(to_string(level).size()), to_string(level).data(),
                     static_cast<int>(msg.size()), msg.data(), loc.file_name(),
                     static_cast<unsigned>(loc.line()));
    }

private:
    Logger() = default;
    std::mutex mu_;
    LogLevel level_ = LogLevel::kInfo;
};

// ---------------------------------------------------------------------------
// Result<T, E>
// ---------------------------------------------------------------------------

/// Wrapper marking a value as an error (std::unexpected before C++23).
template <typename E>
class Unexpected {
public:
    constexpr explicit Unexpected(E e) : error_(std::move(e)) {}
    [[nodiscard]] constexpr const E& error() const& noexcept { return error_; }
    [[nodiscard]] constexpr E& error() & noexcept { return error_; }

private:
    E error_;
};

template <typename E>
[[nodiscard]] constexpr Unexpected<std::decay_t<E>> unexpected(E&& e) {
    return Unexpected<std::decay_t<E>>(std::forward<E>(e));
}

/// Holds either a value of type T or an error of type E.
template <typename T, typename E>
class Result {
public:
    constexpr Result(const T& v) : ok_(true) { new (&storage_.value) T(v); }
    constexpr Result(T&& v) : ok_(true) { new (&storage_.value) T(std::move(v)); }
    constexpr Result(Unexpected<E> u) : ok_(false) { new (&storage_.error) E(std::move(u.error())); }
    Result(const Result& o) : ok_(o.ok_) {
        if (ok_) new (&storage_.value) T(o.storage_.value);
        else new (&storage_.error) E(o.storage_.error);
    }
    Result(Result&& o) noexcept : ok_(o.ok_) {
        if (ok_) new (&storage_.value) T(std::move(o.storage_.value));
        else new (&storage_.error) E(std::move(o.storage_.error));
    }
    Result& operator=(Result o) {
        this->~Result();
        new (this) Result(std::move(o));
        return *this;
    }
    ~Result() {
        if (ok_) storage_.value.~T();
        else storage_.error.~E();
    }

    [[nodiscard]] constexpr bool has_value() const noexcept { return ok_; }
    constexpr explicit operator bool() const noexcept { return ok_; }

    [[nodiscard]] T& value() & {
        TENSORBIT_CHECK(ok_, "Result::value() on an error");
        return storage_.value;
    }
    [[nodiscard]] const T& value() const& {
        TENSORBIT_CHECK(ok_, "Result::value() on an error");
        return storage_.value;
    }
    [[nodiscard]] T&& value() && {
        TENSORBIT_CHECK(ok_, "Result::value() on an error");
        return std::move(storage_.value);
    }
    [[nodiscard]] const E& error() const& {
        TENSORBIT_CHECK(!ok_, "Result::error() on a value");
        return storage_.error;
    }
    [[nodiscard]] T value_or(T alt) const& { return ok_ ? storage_.value : alt; }

    T& operator*() & { return value(); }
    const T& operator*() const& { return value(); }
    T* operator->() { return &value(); }
    const T* operator->() const { return &value(); }

private:
    union Storage {
        Storage() {}
        ~Storage() {}
        T value;
        E error;
    } storage_;
    bool ok_;
};

/// Success-or-error without a value.
template <typename E>
class Result<void, E> {
public:
    constexpr Result() : ok_(true), error_{} {}
    constexpr Result(Unexpected<E> u) : ok_(false), error_(std::move(u.error())) {}
    [[nodiscard]] constexpr bool has_value() const noexcept { return ok_; }
    constexpr explicit operator bool() const noexcept { return ok_; }
    void value() const { TENSORBIT_CHECK(ok_, "Result::value() on an error"); }
    [[nodiscard]] const E& error() const& {
        TENSORBIT_CHECK(!ok_, "Result::error() on a value");
        return error_;
    }

private:
    bool ok_;
    E error_;
};

}  // namespace tensorbit::core

// ---------------------------------------------------------------------------
// Logging macros (common.hpp:383-417); arguments may be rvalues here.
// ---------------------------------------------------------------------------
#define TENSORBIT_LOG_AT(lvl, ...) \
    ::tensorbit::core::Logger::instance().log((lvl), std::format(__VA_ARGS__))
#define TENSORBIT_LOG_TRACE(...) TENSORBIT_LOG_AT(::tensorbit::core::LogLevel::kTrace, __VA_ARGS__)
#define TENSORBIT_LOG_DEBUG(...) TENSORBIT_LOG_AT(::tensorbit::core::LogLevel::kDebug, __VA_ARGS__)
#define TENSORBIT_LOG_INFO(...) TENSORBIT_LOG_AT(::tensorbit::core::LogLevel::kInfo, __VA_ARGS__)
#define TENSORBIT_LOG_WARN(...) TENSORBIT_LOG_AT(::tensorbit::core::LogLevel::kWarn, __VA_ARGS__)
#define TENSORBIT_LOG_ERROR(...) TENSORBIT_LOG_AT(::tensorbit::core::LogLevel::kError, __VA_ARGS__)
#define TENSORBIT_LOG_FATAL(...) TENSORBIT_LOG_AT(::tensorbit::core::LogLevel::kFatal, __VA_ARGS__)
