func.func @column_reduce(%input: memref<8x8xf32>, %output: memref<1x8xf32>) attributes {xt.grid = array<i32: 1, 1, 1>} {
  %zero = arith.constant 0 : i32

  %x = xt.load(%input, %zero, %zero) : (memref<8x8xf32>, i32, i32) -> tensor<8x8xf32>
  %row_sum = xt.reduce_sum(%x) {axis = 0 : i64} : tensor<8x8xf32> -> tensor<1x8xf32>
  xt.store(%row_sum, %output, %zero, %zero) : (tensor<1x8xf32>, memref<1x8xf32>, i32, i32) -> ()
  func.return
}
