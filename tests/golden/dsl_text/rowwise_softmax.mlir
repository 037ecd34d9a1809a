func.func @rowwise_softmax(%input: memref<128x64xf32>, %output: memref<128x64xf32>) attributes {xt.grid = array<i32: 2, 1, 1>, xt.double_buffering = 1 : i32} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32

  %x = xt.load(%input, %bid#0, %zero) : (memref<128x64xf32>, i32, i32) -> tensor<64x64xf32>
  %row_max = xt.reduce_max(%x) {axis = 1 : i64} : tensor<64x64xf32> -> tensor<64x1xf32>
  %shifted = xt.sub(%x, %row_max) : tensor<64x64xf32>, tensor<64x1xf32> -> tensor<64x64xf32>
  %exp = xt.exp(%shifted) : tensor<64x64xf32> -> tensor<64x64xf32>
  %row_sum = xt.reduce_sum(%exp) {axis = 1 : i64} : tensor<64x64xf32> -> tensor<64x1xf32>
  %inv_sum = xt.reciprocal(%row_sum) : tensor<64x1xf32> -> tensor<64x1xf32>
  %normalized = xt.mul(%exp, %inv_sum) : tensor<64x64xf32>, tensor<64x1xf32> -> tensor<64x64xf32>
  xt.store(%normalized, %output, %bid#0, %zero) : (tensor<64x64xf32>, memref<128x64xf32>, i32, i32) -> ()
  func.return
}
