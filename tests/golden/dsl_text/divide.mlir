func.func @divide_kernel(%input: memref<8x8xf32>, %input2: memref<8x1xf32>, %output: memref<8x8xf32>) attributes {xt.grid = array<i32: 1, 1, 1>} {
  %zero = arith.constant 0 : i32

  %x = xt.load(%input, %zero, %zero) : (memref<8x8xf32>, i32, i32) -> tensor<8x8xf32>
  %x2 = xt.load(%input2, %zero, %zero) : (memref<8x1xf32>, i32, i32) -> tensor<8x1xf32>
  %inv_sum = xt.reciprocal(%x2) : tensor<8x1xf32> -> tensor<8x1xf32>
  %normalized = xt.mul(%x, %inv_sum) : tensor<8x8xf32>, tensor<8x1xf32> -> tensor<8x8xf32>
  xt.store(%normalized, %output, %zero, %zero) : (tensor<8x8xf32>, memref<8x8xf32>, i32, i32) -> ()
  func.return
}
