func.func @conv2d_i8(%input: memref<1x32x64x128xi8>, %input2: memref<3x3x128x64xi8>, %output: memref<1x32x64x64xf32>) attributes {xt.grid = array<i32: 1, 1, 1>, xt.double_buffering = 1 : i32} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32

  %x = xt.load(%input2, %zero, %zero, %zero, %zero) {shared = 2 : i64} : (memref<3x3x128x64xi8>, i32, i32, i32, i32) -> tensor<3x3x128x64xi8>
  %load_conv = xt.load_conv2d(%input, %x, %bid#0, %bid#1, %bid#2, %zero) {dilation = array<i64: 1, 1>, group = 1 : i64, pad = array<i64: 1, 1, 1, 1>, stride = array<i64: 1, 1>} : (memref<1x32x64x128xi8>, tensor<3x3x128x64xi8>, i32, i32, i32, i32) -> tensor<1x32x64x64xf32>
  xt.store(%load_conv, %output, %bid#0, %bid#1, %bid#2, %zero) : (tensor<1x32x64x64xf32>, memref<1x32x64x64xf32>, i32, i32, i32, i32) -> ()
  func.return
}
