func.func @mixed(%buf: memref<16x16xf32>, %input: memref<16x16xf32>, %unused: memref<4x4xf32>, %output: memref<16x16xf32>) attributes {xt.grid = array<i32: 1, 1, 1>, xt.double_buffering = 1 : i32} {
  %zero = arith.constant 0 : i32
  %c1 = arith.constant 1 : i32
  %c2 = arith.constant 2 : i32
  %c3 = arith.constant 3 : i32

  %x = xt.load(%buf, %c1, %c2) : (memref<16x16xf32>, i32, i32) -> tensor<4x4xf32>
  %x2 = xt.load(%input, %c3, %c2) : (memref<16x16xf32>, i32, i32) -> tensor<4x4xf32>
  %sum = xt.add(%x, %x2) : tensor<4x4xf32>, tensor<4x4xf32> -> tensor<4x4xf32>
  %shifted = xt.sub(%x, %x2) : tensor<4x4xf32>, tensor<4x4xf32> -> tensor<4x4xf32>
  %sum2 = xt.add(%sum, %shifted) : tensor<4x4xf32>, tensor<4x4xf32> -> tensor<4x4xf32>
  %normalized = xt.mul(%sum2, %sum2) : tensor<4x4xf32>, tensor<4x4xf32> -> tensor<4x4xf32>
  xt.store(%normalized, %buf, %zero, %zero) : (tensor<4x4xf32>, memref<16x16xf32>, i32, i32) -> ()
  %exp = xt.exp(%sum2) : tensor<4x4xf32> -> tensor<4x4xf32>
  xt.store(%exp, %output, %c2, %c1) : (tensor<4x4xf32>, memref<16x16xf32>, i32, i32) -> ()
  func.return
}
