func.func @matmul_kloop(%input: memref<512x512xf32>, %input2: memref<512x512xf32>, %output: memref<512x512xf32>) attributes {xt.grid = array<i32: 4, 4, 1>, xt.double_buffering = 1 : i32} {
  %bid:3 = xt.get_tile_block_id : i32, i32, i32
  %zero = arith.constant 0 : i32
  %c1 = arith.constant 1 : i32
  %c2 = arith.constant 2 : i32
  %c3 = arith.constant 3 : i32
  %c4 = arith.constant 4 : i32
  %c5 = arith.constant 5 : i32
  %c6 = arith.constant 6 : i32
  %c7 = arith.constant 7 : i32

  %x = xt.load(%input, %bid#0, %zero) : (memref<512x512xf32>, i32, i32) -> tensor<128x64xf32>
  %x2 = xt.load(%input2, %zero, %bid#1) : (memref<512x512xf32>, i32, i32) -> tensor<64x128xf32>
  %matmul = xt.matmul(%x, %x2) : tensor<128x64xf32>, tensor<64x128xf32> -> tensor<128x128xf32>
  %x3 = xt.load(%input, %bid#0, %c1) : (memref<512x512xf32>, i32, i32) -> tensor<128x64xf32>
  %x4 = xt.load(%input2, %c1, %bid#1) : (memref<512x512xf32>, i32, i32) -> tensor<64x128xf32>
  %matmul2 = xt.matmul(%x3, %x4) : tensor<128x64xf32>, tensor<64x128xf32> -> tensor<128x128xf32>
  %sum = xt.add(%matmul, %matmul2) : tensor<128x128xf32>, tensor<128x128xf32> -> tensor<128x128xf32>
  %x5 = xt.load(%input, %bid#0, %c2) : (memref<512x512xf32>, i32, i32) -> tensor<128x64xf32>
  %x6 = xt.load(%input2, %c2, %bid#1) : (memref<512x512xf32>, i32, i32) -> tensor<64x128xf32>
  %matmul3 = xt.matmul(%x5, %x6) : tensor<128x64xf32>, tensor<64x128xf32> -> tensor<128x128xf32>
  %sum2 = xt.add(%sum, %matmul3) : tensor<128x128xf32>, tensor<128x128xf32> -> tensor<128x128xf32>
  %x7 = xt.load(%input, %bid#0, %c3) : (memref<512x512xf32>, i32, i32) -> tensor<128x64xf32>
  %x8 = xt.load(%input2, %c3, %bid#1) : (memref<512x512xf32>, i32, i32) -> tensor<64x128xf32>
  %matmul4 = xt.matmul(%x7, %x8) : tensor<128x64xf32>, tensor<64x128xf32> -> tensor<128x128xf32>
  %sum3 = xt.add(%sum2, %matmul4) : tensor<128x128xf32>, tensor<128x128xf32> -> tensor<128x128xf32>
  %x9 = xt.load(%input, %bid#0, %c4) : (memref<512x512xf32>, i32, i32) -> tensor<128x64xf32>
  %x10 = xt.load(%input2, %c4, %bid#1) : (memref<512x512xf32>, i32, i32) -> tensor<64x128xf32>
  %matmul5 = xt.matmul(%x9, %x10) : tensor<128x64xf32>, tensor<64x128xf32> -> tensor<128x128xf32>
  %sum4 = xt.add(%sum3, %matmul5) : tensor<128x128xf32>, tensor<128x128xf32> -> tensor<128x128xf32>
  %x11 = xt.load(%input, %bid#0, %c5) : (memref<512x512xf32>, i32, i32) -> tensor<128x64xf32>
  %x12 = xt.load(%input2, %c5, %bid#1) : (memref<512x512xf32>, i32, i32) -> tensor<64x128xf32>
  %matmul6 = xt.matmul(%x11, %x12) : tensor<128x64xf32>, tensor<64x128xf32> -> tensor<128x128xf32>
  %sum5 = xt.add(%sum4, %matmul6) : tensor<128x128xf32>, tensor<128x128xf32> -> tensor<128x128xf32>
  %x13 = xt.load(%input, %bid#0, %c6) : (memref<512x512xf32>, i32, i32) -> tensor<128x64xf32>
  %x14 = xt.load(%input2, %c6, %bid#1) : (memref<512x512xf32>, i32, i32) -> tensor<64x128xf32>
  %matmul7 = xt.matmul(%x13, %x14) : tensor<128x64xf32>, tensor<64x128xf32> -> tensor<128x128xf32>
  %sum6 = xt.add(%sum5, %matmul7) : tensor<128x128xf32>, tensor<128x128xf32> -> tensor<128x128xf32>
  %x15 = xt.load(%input, %bid#0, %c7) : (memref<512x512xf32>, i32, i32) -> tensor<128x64xf32>
  %x16 = xt.load(%input2, %c7, %bid#1) : (memref<512x512xf32>, i32, i32) -> tensor<64x128xf32>
  %matmul8 = xt.matmul(%x15, %x16) : tensor<128x64xf32>, tensor<64x128xf32> -> tensor<128x128xf32>
  %sum7 = xt.add(%sum6, %matmul8) : tensor<128x128xf32>, tensor<128x128xf32> -> tensor<128x128xf32>
  xt.store(%sum7, %output, %bid#0, %bid#1) : (tensor<128x128xf32>, memref<512x512xf32>, i32, i32) -> ()
  func.return
}
