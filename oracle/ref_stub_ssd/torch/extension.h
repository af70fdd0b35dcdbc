/* TEST INFRASTRUCTURE ONLY.  Stand-in for <torch/extension.h> when the
 * reference's csrc/transfer_ssd.cpp is compiled as the SSD-tier oracle:
 * that file only reads raw pointers and lengths out of 1-D tensors
 * (data_ptr<T>(), size(0)), so a two-field view replaces libtorch, and the
 * standard headers the reference gets through torch are included here. */
#pragma once
#include <cstddef>
#include <cstdint>
#include <cstdio>
#include <iostream>
#include <map>
#include <stdexcept>
#include <string>
#include <vector>

namespace torch {
class Tensor {
 public:
  Tensor(void *data, int64_t numel) : data_(data), numel_(numel) {}
  template <typename T>
  T *data_ptr() const { return static_cast<T *>(data_); }
  int64_t size(int) const { return numel_; }

 private:
  void *data_;
  int64_t numel_;
};
}  // namespace torch
