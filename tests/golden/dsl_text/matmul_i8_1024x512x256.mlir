func.func @matmul_i8(%input: memref<1024x256xi8>, %input2: memref<256x512xi8>, %output: memref<1024x512xi8>, %input3: memref<1x512xf32>, %input4: memref<1x512xf32>) attributes {xt.grid = array<i32: 16, 8, 1>, xt.double_buffering = 1 : i32} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32

  %x = xt.load(%input, %bid#0, %zero) : (memref<1024x256xi8>, i32, i32) -> tensor<64x256xi8>
  %x2 = xt.load(%input2, %zero, %bid#1) {shared = 1 : i64} : (memref<256x512xi8>, i32, i32) -> tensor<256x64xi8>
  %x3 = xt.load(%input3, %zero, %bid#1) {shared = 1 : i64} : (memref<1x512xf32>, i32, i32) -> tensor<1x64xf32>
  %x4 = xt.load(%input4, %zero, %bid#1) {shared = 1 : i64} : (memref<1x512xf32>, i32, i32) -> tensor<1x64xf32>
  %matmul = xt.matmul(%x, %x2) : tensor<64x256xi8>, tensor<256x64xi8> -> tensor<64x64xf32>
  %normalized = xt.mul(%matmul, %x3) : tensor<64x64xf32>, tensor<1x64xf32> -> tensor<64x64xf32>
  %sum = xt.add(%normalized, %x4) : tensor<64x64xf32>, tensor<1x64xf32> -> tensor<64x64xf32>
  %cast = xt.ftoi(%sum) : tensor<64x64xf32> -> tensor<64x64xi8>
  xt.store(%cast, %output, %bid#0, %bid#1) : (tensor<64x64xi8>, memref<1024x512xi8>, i32, i32) -> ()
  func.return
}
