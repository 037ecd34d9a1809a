func.func @compute_mma(%input: memref<16x32xi8>, %input2: memref<32x8xi8>, %input3: memref<16x8xf32>, %output: memref<16x8xf32>) attributes {xt.grid = array<i32: 1, 1, 1>} {
  %zero = arith.constant 0 : i32

  %x = xt.load(%input, %zero, %zero) : (memref<16x32xi8>, i32, i32) -> tensor<16x32xi8>
  %x2 = xt.load(%input2, %zero, %zero) : (memref<32x8xi8>, i32, i32) -> tensor<32x8xi8>
  %x3 = xt.load(%input3, %zero, %zero) : (memref<16x8xf32>, i32, i32) -> tensor<16x8xf32>
  %mma = xt.mma(%x, %x2, %x3) : tensor<16x32xi8>, tensor<32x8xi8>, tensor<16x8xf32> -> tensor<16x8xf32>
  xt.store(%mma, %output, %zero, %zero) : (tensor<16x8xf32>, memref<16x8xf32>, i32, i32) -> ()
  func.return
}
