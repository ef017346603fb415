// block_pool.h -- host bookkeeping of paged KV blocks.
//
// Behaves like the reference's BlockPool / BlockTable
// (gpu-engine/include/engine/kv_cache.h:16-57, gpu-engine/src/kv_cache_pool.cpp:6-28):
// a LIFO stack of free block ids (the first allocation returns 0, a freed id
// is the next one handed out), allocate() returns -1 when nothing is free,
// free() throws std::out_of_range for an id outside the pool and
// std::logic_error for an id that is not allocated.  The allocator's policy is
// part of the contract the scheduler sees (free_blocks() drives admission),
// so it is kept identical.
#pragma once

#include <stdexcept>
#include <string>
#include <vector>

namespace b2 {

class BlockPool {
public:
    explicit BlockPool(int num_blocks) : num_blocks_(num_blocks), in_use_(static_cast<size_t>(num_blocks), 0) {
        free_.reserve(static_cast<size_t>(num_blocks));
        for (int id = num_blocks - 1; id >= 0; --id) free_.push_back(id);
    }

    int allocate() {
        if (free_.empty()) return -1;
        const int id = free_.back();
        free_.pop_back();
        in_use_[static_cast<size_t>(id)] = 1;
        return id;
    }

    void free(int id) {
        if (id < 0 || id >= num_blocks_) throw std::out_of_range("BlockPool::free: block id " + std::to_string(id) + " out of range");
        if (!in_use_[static_cast<size_t>(id)]) throw std::logic_error("BlockPool::free: block id " + std::to_string(id) + " is not allocated");
        in_use_[static_cast<size_t>(id)] = 0;
        free_.push_back(id);
    }

    int num_free() const { return static_cast<int>(free_.size()); }
    int num_total() const { return num_blocks_; }

private:
    int num_blocks_;
    std::vector<int> free_;
    std::vector<char> in_use_;
};

// Block ids of one sequence in allocation order; entry i covers positions
// [16 i, 16 i + 16).
struct BlockTable {
    std::vector<int> ids;
};

}  // namespace b2
