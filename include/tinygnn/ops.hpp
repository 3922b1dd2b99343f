// ============================================================================
//  tinygnn/ops.hpp -- TinyGNN's operators on device tensors.
//
//  Same declarations and exceptions as the reference's include/tinygnn/
//  ops.hpp:76-286; each call runs the matching sm_100a kernel through the C
//  ABI (include/tinygnn_b200.h) on the calling thread's default stream.
// ============================================================================
#pragma once

#include "tinygnn/tensor.hpp"

namespace tinygnn {

Tensor matmul(const Tensor& A, const Tensor& B);              // ops.hpp:76
Tensor spmm(const Tensor& A, const Tensor& B);                // ops.hpp:112
void relu_inplace(Tensor& X);                                 // ops.hpp:132
void leaky_relu_inplace(Tensor& X, float alpha = 0.01f);      // ops.hpp:149
void elu_inplace(Tensor& X, float alpha = 1.0f);              // ops.hpp:166
void sigmoid_inplace(Tensor& X);                              // ops.hpp:186
void tanh_inplace(Tensor& X);                                 // ops.hpp:202
void gelu_inplace(Tensor& X);                                 // ops.hpp:219
void softmax_inplace(Tensor& X);                              // ops.hpp:242
void log_softmax_inplace(Tensor& X);                          // ops.hpp:262
void add_bias(Tensor& X, const Tensor& bias);                 // ops.hpp:286

}  // namespace tinygnn
