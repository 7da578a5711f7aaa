// hls_stream.h -- minimal FIFO used ONLY to compile the reference VectorOP
// kernel (kernels/vectorop/kernel/VectorOP.cpp) for CPU C-simulation as a
// parity checker.  Test infrastructure, not product code.
//
// In C-simulation the reference's dataflow stages run one after another
// (load_a, load_b, compute, store_c), so an unbounded FIFO reproduces the
// element order exactly.  Reading an empty stream returns a value-initialised
// element instead of aborting.
#pragma once

#include <cstddef>
#include <deque>

namespace hls {

template <typename T>
class stream {
public:
    stream() {}
    explicit stream(const char*) {}
    void write(const T& v) { q_.push_back(v); }
    T read() {
        if (q_.empty()) return T();
        T v = q_.front();
        q_.pop_front();
        return v;
    }
    void operator<<(const T& v) { write(v); }
    void operator>>(T& v) { v = read(); }
    bool empty() const { return q_.empty(); }
    bool full() const { return false; }
    std::size_t size() const { return q_.size(); }

private:
    std::deque<T> q_;
};

}  // namespace hls
