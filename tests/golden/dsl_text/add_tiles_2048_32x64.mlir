func.func @add_tiles(%input: memref<2048x2048xf32>, %input2: memref<2048x2048xf32>, %output: memref<2048x2048xf32>) attributes {xt.grid = array<i32: 64, 32, 1>, xt.double_buffering = 1 : i32} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %x = xt.load(%input, %bid#0, %bid#1) : (memref<2048x2048xf32>, i32, i32) -> tensor<32x64xf32>
  %x2 = xt.load(%input2, %bid#0, %bid#1) : (memref<2048x2048xf32>, i32, i32) -> tensor<32x64xf32>
  %sum = xt.add(%x, %x2) : tensor<32x64xf32>, tensor<32x64xf32> -> tensor<32x64xf32>
  xt.store(%sum, %output, %bid#0, %bid#1) : (tensor<32x64xf32>, memref<2048x2048xf32>, i32, i32) -> ()
  func.return
}
