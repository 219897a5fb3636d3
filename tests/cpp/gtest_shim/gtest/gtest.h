// gtest.h — a minimal GoogleTest-compatible header (GTest is not installed here).
//
// Implements what the op tests use: ::testing::Test fixtures, TEST_F, EXPECT_NEAR,
// EXPECT_TRUE, ASSERT_EQ, ASSERT_TRUE with streamed messages, SCOPED_TRACE,
// InitGoogleTest and RUN_ALL_TESTS.  Failures print file:line, the active traces and
// the streamed message (the first 20 per test); RUN_ALL_TESTS returns non-zero when a
// test failed.
#pragma once

#include <cmath>
#include <cstdio>
#include <functional>
#include <sstream>
#include <string>
#include <vector>

namespace testing {

class Test {
public:
    virtual ~Test() = default;
    virtual void SetUp() {}
    virtual void TearDown() {}
    virtual void TestBody() = 0;
};

class Message {
public:
    template <class T>
    Message &operator<<(const T &v)
    {
        ss_ << v;
        return *this;
    }
    std::string str() const { return ss_.str(); }

private:
    std::ostringstream ss_;
};

namespace internal {

struct Registered {
    std::string suite, name;
    std::function<Test *()> make;
};

inline std::vector<Registered> &registry()
{
    static std::vector<Registered> r;
    return r;
}

struct State {
    int failures = 0;
    std::vector<std::string> traces;
};

inline State &state()
{
    static State s;
    return s;
}

inline bool Register(const char *suite, const char *name, std::function<Test *()> make)
{
    registry().push_back({suite, name, std::move(make)});
    return true;
}

class AssertHelper {
public:
    AssertHelper(const char *file, int line, std::string what) : file_(file), line_(line), what_(std::move(what)) {}
    void operator=(const Message &m) const
    {
        State &s = state();
        if (s.failures++ < 20) {
            std::printf("%s:%d: Failure: %s\n", file_, line_, what_.c_str());
            for (const auto &t : s.traces) std::printf("  trace: %s\n", t.c_str());
            const std::string msg = m.str();
            if (!msg.empty()) std::printf("  %s\n", msg.c_str());
        }
    }

private:
    const char *file_;
    int line_;
    std::string what_;
};

class ScopedTrace {
public:
    explicit ScopedTrace(const std::string &msg) { state().traces.push_back(msg); }
    ~ScopedTrace() { state().traces.pop_back(); }
};

inline std::string near_text(double a, double b, double tol)
{
    std::ostringstream ss;
    ss << "|" << a << " - " << b << "| > " << tol;
    return ss.str();
}

inline int RunAll()
{
    int failed_tests = 0;
    for (const auto &r : registry()) {
        std::printf("[ RUN      ] %s.%s\n", r.suite.c_str(), r.name.c_str());
        const int before = state().failures;
        Test *t = r.make();
        t->SetUp();
        t->TestBody();
        t->TearDown();
        delete t;
        const bool ok = state().failures == before;
        failed_tests += ok ? 0 : 1;
        std::printf("[ %s ] %s.%s (%d failures)\n", ok ? "      OK" : " FAILED ", r.suite.c_str(), r.name.c_str(),
                    state().failures - before);
    }
    std::printf("[==========] %zu tests ran, %d failed\n", registry().size(), failed_tests);
    return failed_tests ? 1 : 0;
}

}  // namespace internal

inline void InitGoogleTest(int *, char **) {}

}  // namespace testing

#define TEST_F(fixture, name)                                                                               \
    class fixture##_##name##_Test : public fixture {                                                        \
    public:                                                                                                 \
        void TestBody() override;                                                                           \
    };                                                                                                      \
    static const bool fixture##_##name##_registered =                                                       \
        ::testing::internal::Register(#fixture, #name, []() -> ::testing::Test * { return new fixture##_##name##_Test; }); \
    void fixture##_##name##_Test::TestBody()

#define EXPECT_NEAR(a, b, tol)                                                                              \
    if (std::fabs(static_cast<double>(a) - static_cast<double>(b)) <= static_cast<double>(tol))             \
        ;                                                                                                   \
    else                                                                                                    \
        ::testing::internal::AssertHelper(__FILE__, __LINE__,                                               \
                                          ::testing::internal::near_text((a), (b), (tol))) = ::testing::Message()

#define EXPECT_TRUE(c) \
    if (c)             \
        ;              \
    else               \
        ::testing::internal::AssertHelper(__FILE__, __LINE__, "EXPECT_TRUE(" #c ")") = ::testing::Message()

#define ASSERT_TRUE(c) \
    if (c)             \
        ;              \
    else               \
        return ::testing::internal::AssertHelper(__FILE__, __LINE__, "ASSERT_TRUE(" #c ")") = ::testing::Message()

#define ASSERT_EQ(a, b)  \
    if ((a) == (b))      \
        ;                \
    else                 \
        return ::testing::internal::AssertHelper(__FILE__, __LINE__, "ASSERT_EQ(" #a ", " #b ")") = ::testing::Message()

#define FE_GTEST_CAT2(a, b) a##b
#define FE_GTEST_CAT(a, b) FE_GTEST_CAT2(a, b)
#define SCOPED_TRACE(msg) ::testing::internal::ScopedTrace FE_GTEST_CAT(fe_gtest_trace_, __LINE__)(msg)

#define RUN_ALL_TESTS() ::testing::internal::RunAll()
