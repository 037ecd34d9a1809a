func.func @unary_and_shape(%input: memref<8x8xf32>, %output: memref<8x8xf32>, %output2: memref<4x16xf32>, %input2: memref<2x3x4xf32>, %output3: memref<2x4x3xf32>) attributes {xt.grid = array<i32: 1, 1, 1>} {
  %zero = arith.constant 0 : i32

  %x = xt.load(%input, %zero, %zero) : (memref<8x8xf32>, i32, i32) -> tensor<8x8xf32>
  %cos = xt.cos(%x) : tensor<8x8xf32> -> tensor<8x8xf32>
  %sin = xt.sin(%cos) : tensor<8x8xf32> -> tensor<8x8xf32>
  %rsqrt = xt.rsqrt(%sin) : tensor<8x8xf32> -> tensor<8x8xf32>
  %sigmoid = xt.sigmoid(%rsqrt) : tensor<8x8xf32> -> tensor<8x8xf32>
  %tanh = xt.tanh(%sigmoid) : tensor<8x8xf32> -> tensor<8x8xf32>
  %silu = xt.silu(%tanh) : tensor<8x8xf32> -> tensor<8x8xf32>
  xt.store(%silu, %output, %zero, %zero) : (tensor<8x8xf32>, memref<8x8xf32>, i32, i32) -> ()
  %reshape = xt.reshape(%silu) : tensor<8x8xf32> -> tensor<4x16xf32>
  xt.store(%reshape, %output2, %zero, %zero) : (tensor<4x16xf32>, memref<4x16xf32>, i32, i32) -> ()
  %x2 = xt.load(%input2, %zero, %zero, %zero) : (memref<2x3x4xf32>, i32, i32, i32) -> tensor<2x3x4xf32>
  %transpose = xt.transpose(%x2) : tensor<2x3x4xf32> -> tensor<2x4x3xf32>
  xt.store(%transpose, %output3, %zero, %zero, %zero) : (tensor<2x4x3xf32>, memref<2x4x3xf32>, i32, i32, i32) -> ()
  func.return
}
