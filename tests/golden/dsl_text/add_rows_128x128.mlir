func.func @add_rows(%input: memref<128x128xf32>, %input2: memref<128x128xf32>, %output: memref<128x128xf32>) attributes {xt.grid = array<i32: 2, 1, 1>, xt.double_buffering = 1 : i32} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32

  %x = xt.load(%input, %bid#0, %zero) : (memref<128x128xf32>, i32, i32) -> tensor<64x128xf32>
  %x2 = xt.load(%input2, %bid#0, %zero) : (memref<128x128xf32>, i32, i32) -> tensor<64x128xf32>
  %sum = xt.add(%x, %x2) : tensor<64x128xf32>, tensor<64x128xf32> -> tensor<64x128xf32>
  xt.store(%sum, %output, %bid#0, %zero) : (tensor<64x128xf32>, memref<128x128xf32>, i32, i32) -> ()
  func.return
}
