// spmd.kernel functions in the dialect's generic form, used by the shim tests.

func.func @ewise(%A: memref<?xf32>, %B: memref<?xf32>, %C: memref<?xf32>, %N: index)
    attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %a = memref.load %A[%i] : memref<?xf32>
    %b = memref.load %B[%i] : memref<?xf32>
    %s = arith.addf %a, %b : f32
    memref.store %s, %C[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>,
      "spmd.tile_sizes" = array<i64: 32>} : (index, index, index) -> ()
  func.return
}

func.func @axpy(%X: memref<?xf32>, %Y: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %alpha = arith.constant 2.5 : f32
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %x = memref.load %X[%i] : memref<?xf32>
    %y = memref.load %Y[%i] : memref<?xf32>
    %ax = arith.mulf %alpha, %x : f32
    %r = arith.addf %ax, %y : f32
    memref.store %r, %Y[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>} : (index, index, index) -> ()
  func.return
}

func.func @promoted_stencil(%A: memref<?x?xf32>, %B: memref<?x?xf32>, %N: index, %M: index)
    attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c8 = arith.constant 8 : index
  %c32 = arith.constant 32 : index
  "spmd.forall"(%c0, %c0, %N, %M, %c32, %c8) ({
  ^bb0(%ii: index, %jj: index):
    "spmd.forall"(%c0, %c0, %c32, %c8, %c1, %c1) ({
    ^bb0(%ti: index, %tj: index):
      %i = arith.addi %ii, %ti : index
      %j = arith.addi %jj, %tj : index
      %ip = arith.addi %i, %c1 : index
      %jp = arith.addi %j, %c1 : index
      %x0 = memref.load %A[%i, %j] : memref<?x?xf32>
      %x1 = memref.load %A[%i, %jp] : memref<?x?xf32>
      %x2 = memref.load %A[%ip, %j] : memref<?x?xf32>
      %s0 = arith.addf %x0, %x1 : f32
      %s1 = arith.addf %s0, %x2 : f32
      memref.store %s1, %B[%i, %j] : memref<?x?xf32>
      "spmd.yield"() : () -> ()
    }) {operandSegmentSizes = array<i32: 2, 2, 2>, "spmd.mapping" = #spmd.level<lane>}
       : (index, index, index, index, index, index) -> ()
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 2, 2, 2>, "spmd.mapping" = #spmd.level<group>,
      "spmd.tile_sizes" = array<i64: 32, 8>, "spmd.memory_policy" = #spmd.memory_policy<prefer_group>}
     : (index, index, index, index, index, index) -> ()
  func.return
}

func.func @jacobi_interior(%U: memref<?x?xf32>, %V: memref<?x?xf32>, %N: index, %M: index)
    attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c16 = arith.constant 16 : index
  %c32 = arith.constant 32 : index
  %k = arith.constant 0.2 : f32
  "spmd.forall"(%c0, %c0, %N, %M, %c16, %c32) ({
  ^bb0(%ii: index, %jj: index):
    "spmd.forall"(%c0, %c0, %c16, %c32, %c1, %c1) ({
    ^bb0(%ti: index, %tj: index):
      %i = arith.addi %ii, %ti : index
      %j = arith.addi %jj, %tj : index
      %in = arith.subi %i, %c1 : index
      %is = arith.addi %i, %c1 : index
      %je = arith.addi %j, %c1 : index
      %jw = arith.subi %j, %c1 : index
      %c = memref.load %U[%i, %j] : memref<?x?xf32>
      %n = memref.load %U[%in, %j] : memref<?x?xf32>
      %s = memref.load %U[%is, %j] : memref<?x?xf32>
      %e = memref.load %U[%i, %je] : memref<?x?xf32>
      %w = memref.load %U[%i, %jw] : memref<?x?xf32>
      %t0 = arith.addf %c, %n : f32
      %t1 = arith.addf %t0, %s : f32
      %t2 = arith.addf %t1, %e : f32
      %t3 = arith.addf %t2, %w : f32
      %o = arith.mulf %t3, %k : f32
      memref.store %o, %V[%i, %j] : memref<?x?xf32>
      "spmd.yield"() : () -> ()
    }) {operandSegmentSizes = array<i32: 2, 2, 2>, "spmd.mapping" = #spmd.level<lane>}
       : (index, index, index, index, index, index) -> ()
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 2, 2, 2>, "spmd.mapping" = #spmd.level<group>,
      "spmd.tile_sizes" = array<i64: 16, 32>, "spmd.memory_policy" = #spmd.memory_policy<prefer_group>}
     : (index, index, index, index, index, index) -> ()
  func.return
}

func.func @pairs_stepped(%A: memref<?xf32>, %B: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c2 = arith.constant 2 : index
  %c4 = arith.constant 4 : index
  %c8 = arith.constant 8 : index
  "spmd.forall"(%c0, %N, %c8) ({
  ^bb0(%ii: index):
    "spmd.forall"(%c0, %c4, %c1) ({
    ^bb0(%ti: index):
      %sc = arith.muli %ti, %c2 : index
      %p = arith.addi %ii, %sc : index
      %p1 = arith.addi %p, %c1 : index
      %a0 = memref.load %A[%p] : memref<?xf32>
      %a1 = memref.load %A[%p1] : memref<?xf32>
      %s = arith.addf %a0, %a1 : f32
      memref.store %s, %B[%p] : memref<?xf32>
      "spmd.yield"() : () -> ()
    }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<lane>} : (index, index, index) -> ()
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>,
      "spmd.tile_sizes" = array<i64: 4>, "spmd.memory_policy" = #spmd.memory_policy<prefer_group>}
     : (index, index, index) -> ()
  func.return
}

func.func @hierarchical_sum(%A: memref<?xf32>, %out: memref<f32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c256 = arith.constant 256 : index
  "spmd.forall"(%c0, %N, %c256) ({
  ^bb0(%t0: index):
    %z = arith.constant 0 : index
    %one = arith.constant 1 : index
    %n256 = arith.constant 256 : index
    %zero = arith.constant 0.0 : f32
    %sum = "spmd.reduce"(%z, %n256, %one, %zero) ({
    ^bb1(%l: index):
      %g = arith.addi %t0, %l : index
      %ok = arith.cmpi ult, %g, %N : index
      %gi = arith.select %ok, %g, %z : index
      %x = memref.load %A[%gi] : memref<?xf32>
      %v = arith.select %ok, %x, %zero : f32
      "spmd.yield"(%v) : (f32) -> ()
    }) {"spmd.kind" = #spmd.reduction_kind<add>} : (index, index, index, f32) -> f32
    %old = memref.atomic_rmw addf %sum, %out[] : (f32, memref<f32>) -> f32
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>,
      "spmd.tile_sizes" = array<i64: 256>} : (index, index, index) -> ()
  func.return
}

func.func @max_i32(%A: memref<?xi32>, %out: memref<i32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c128 = arith.constant 128 : index
  "spmd.forall"(%c0, %N, %c128) ({
  ^bb0(%t0: index):
    %z = arith.constant 0 : index
    %lo = arith.constant -2147483648 : i32
    %m = "spmd.reduce"(%z, %c128, %c1, %lo) ({
    ^bb1(%l: index):
      %g = arith.addi %t0, %l : index
      %ok = arith.cmpi ult, %g, %N : index
      %gi = arith.select %ok, %g, %z : index
      %x = memref.load %A[%gi] : memref<?xi32>
      %v = arith.select %ok, %x, %lo : i32
      "spmd.yield"(%v) : (i32) -> ()
    }) {"spmd.kind" = #spmd.reduction_kind<max>} : (index, index, index, i32) -> i32
    %old = memref.atomic_rmw maxs %m, %out[] : (i32, memref<i32>) -> i32
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>} : (index, index, index) -> ()
  func.return
}

func.func @gather_unsupported(%A: memref<?xf32>, %B: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %k = arith.muli %i, %N : index
    %a = memref.load %A[%k] : memref<?xf32>
    memref.store %a, %B[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>} : (index, index, index) -> ()
  func.return
}

func.func @smooth_interior(%A: memref<?xf32>, %B: memref<?xf32>, %Nm1: index) attributes {spmd.kernel} {
  %c1 = arith.constant 1 : index
  %half = arith.constant 0.5 : f32
  "spmd.forall"(%c1, %Nm1, %c1) ({
  ^bb0(%i: index):
    %im = arith.subi %i, %c1 : index
    %ip = arith.addi %i, %c1 : index
    %l = memref.load %A[%im] : memref<?xf32>
    %r = memref.load %A[%ip] : memref<?xf32>
    %hl = arith.mulf %half, %l : f32
    %hr = arith.mulf %half, %r : f32
    %s = arith.addf %hl, %hr : f32
    memref.store %s, %B[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>,
      "spmd.tile_sizes" = array<i64: 64>, "spmd.memory_policy" = #spmd.memory_policy<prefer_group>}
     : (index, index, index) -> ()
  func.return
}

// Elementwise bodies beyond add / axpy (the general forall map).
func.func @mul2d(%A: memref<?x?xf32>, %B: memref<?x?xf32>, %C: memref<?x?xf32>, %N: index, %M: index)
    attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %c0, %N, %M, %c1, %c1) ({
  ^bb0(%i: index, %j: index):
    %a = memref.load %A[%i, %j] : memref<?x?xf32>
    %b = memref.load %B[%i, %j] : memref<?x?xf32>
    %p = arith.mulf %a, %b : f32
    memref.store %p, %C[%i, %j] : memref<?x?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 2, 2, 2>} : (index, index, index, index, index, index) -> ()
  func.return
}

func.func @plus_one_from4(%A: memref<?xf32>, %B: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c4 = arith.constant 4 : index
  %c1 = arith.constant 1 : index
  %one = arith.constant 1.0 : f32
  "spmd.forall"(%c4, %N, %c1) ({
  ^bb0(%i: index):
    %a = memref.load %A[%i] : memref<?xf32>
    %b = arith.addf %a, %one : f32
    memref.store %b, %B[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}

func.func @clamp_tiled(%A: memref<?xf32>, %B: memref<?xf32>, %N: index, %lim: f32) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c128 = arith.constant 128 : index
  "spmd.forall"(%c0, %N, %c128) ({
  ^bb0(%t: index):
    "spmd.forall"(%c0, %c128, %c1) ({
    ^bb1(%l: index):
      %i = arith.addi %t, %l : index
      %a = memref.load %A[%i] : memref<?xf32>
      %big = arith.cmpf ogt, %a, %lim : f32
      %neg = arith.negf %lim : f32
      %small = arith.cmpf olt, %a, %neg : f32
      %hi = arith.select %big, %lim, %a : f32
      %v = arith.select %small, %neg, %hi : f32
      memref.store %v, %B[%i] : memref<?xf32>
      "spmd.yield"() : () -> ()
    }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<lane>} : (index, index, index) -> ()
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>,
      "spmd.tile_sizes" = array<i64: 128>} : (index, index, index) -> ()
  func.return
}

func.func @hypot3d(%X: memref<?x?x?xf32>, %Y: memref<?x?x?xf32>, %R: memref<?x?x?xf32>, %D: index, %H: index,
                   %W: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %c2 = arith.constant 2 : index
  "spmd.forall"(%c0, %c0, %c0, %D, %H, %W, %c1, %c1, %c2) ({
  ^bb0(%i: index, %j: index, %k: index):
    %x = memref.load %X[%i, %j, %k] : memref<?x?x?xf32>
    %y = memref.load %Y[%i, %j, %k] : memref<?x?x?xf32>
    %xx = arith.mulf %x, %x : f32
    %yy = arith.mulf %y, %y : f32
    %s = arith.addf %xx, %yy : f32
    %r = math.sqrt %s : f32
    %ax = math.absf %x : f32
    %m = arith.maximumf %r, %ax : f32
    %d = arith.divf %m, %r : f32
    memref.store %d, %R[%i, %j, %k] : memref<?x?x?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 3, 3, 3>} : (index, index, index, index, index, index, index, index, index) -> ()
  func.return
}

func.func @scale_in_place(%B: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %two = arith.constant 2.0 : f32
  %one = arith.constant 1.0 : f32
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %b = memref.load %B[%i] : memref<?xf32>
    %t = arith.mulf %b, %two : f32
    %u = arith.addf %t, %one : f32
    memref.store %u, %B[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}

// Guarded stores (spmd.if inside an elementwise forall).
func.func @clamp_guarded(%A: memref<?xf32>, %N: index, %t: f32) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %v = memref.load %A[%i] : memref<?xf32>
    %big = arith.cmpf ogt, %v, %t : f32
    "spmd.if"(%big) ({
      memref.store %t, %A[%i] : memref<?xf32>
      "spmd.yield"() : () -> ()
    }, {
      "spmd.yield"() : () -> ()
    }) : (i1) -> ()
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>, "spmd.mapping" = #spmd.level<group>} : (index, index, index) -> ()
  func.return
}

func.func @abs_if_else(%A: memref<?x?xf32>, %B: memref<?x?xf32>, %N: index, %M: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %zero = arith.constant 0.0 : f32
  "spmd.forall"(%c0, %c0, %N, %M, %c1, %c1) ({
  ^bb0(%i: index, %j: index):
    %a = memref.load %A[%i, %j] : memref<?x?xf32>
    %pos = arith.cmpf oge, %a, %zero : f32
    "spmd.if"(%pos) ({
      memref.store %a, %B[%i, %j] : memref<?x?xf32>
      "spmd.yield"() : () -> ()
    }, {
      %n = arith.negf %a : f32
      memref.store %n, %B[%i, %j] : memref<?x?xf32>
      "spmd.yield"() : () -> ()
    }) : (i1) -> ()
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 2, 2, 2>} : (index, index, index, index, index, index) -> ()
  func.return
}

func.func @select_by_if(%A: memref<?xf32>, %B: memref<?xf32>, %C: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c0, %N, %c1) ({
  ^bb0(%i: index):
    %a = memref.load %A[%i] : memref<?xf32>
    %b = memref.load %B[%i] : memref<?xf32>
    %lt = arith.cmpf olt, %a, %b : f32
    %m = "spmd.if"(%lt) ({
      %d = arith.subf %b, %a : f32
      "spmd.yield"(%d) : (f32) -> ()
    }, {
      %e = arith.subf %a, %b : f32
      "spmd.yield"(%e) : (f32) -> ()
    }) : (i1) -> f32
    memref.store %m, %C[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}

// Non-linear stencils: loads at constant offsets are shifted views.
func.func @max_filter_interior(%A: memref<?xf32>, %B: memref<?xf32>, %Nm1: index) attributes {spmd.kernel} {
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c1, %Nm1, %c1) ({
  ^bb0(%i: index):
    %im = arith.subi %i, %c1 : index
    %ip = arith.addi %i, %c1 : index
    %l = memref.load %A[%im] : memref<?xf32>
    %r = memref.load %A[%ip] : memref<?xf32>
    %c = memref.load %A[%i] : memref<?xf32>
    %m = arith.maximumf %l, %r : f32
    %d = arith.subf %m, %c : f32
    memref.store %d, %B[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}

func.func @upwind2d(%A: memref<?x?xf32>, %B: memref<?x?xf32>, %Nm1: index, %M: index) attributes {spmd.kernel} {
  %c0 = arith.constant 0 : index
  %c1 = arith.constant 1 : index
  %zero = arith.constant 0.0 : f32
  "spmd.forall"(%c1, %c0, %Nm1, %M, %c1, %c1) ({
  ^bb0(%i: index, %j: index):
    %im = arith.subi %i, %c1 : index
    %ip = arith.addi %i, %c1 : index
    %c = memref.load %A[%i, %j] : memref<?x?xf32>
    %n = memref.load %A[%im, %j] : memref<?x?xf32>
    %s = memref.load %A[%ip, %j] : memref<?x?xf32>
    %pos = arith.cmpf ogt, %c, %zero : f32
    %back = arith.subf %c, %n : f32
    %fwd = arith.subf %s, %c : f32
    %v = arith.select %pos, %back, %fwd : f32
    memref.store %v, %B[%i, %j] : memref<?x?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 2, 2, 2>} : (index, index, index, index, index, index) -> ()
  func.return
}

func.func @in_place_neighbour_unsupported(%A: memref<?xf32>, %N: index) attributes {spmd.kernel} {
  %c1 = arith.constant 1 : index
  "spmd.forall"(%c1, %N, %c1) ({
  ^bb0(%i: index):
    %im = arith.subi %i, %c1 : index
    %l = memref.load %A[%im] : memref<?xf32>
    %c = memref.load %A[%i] : memref<?xf32>
    %m = arith.maximumf %l, %c : f32
    memref.store %m, %A[%i] : memref<?xf32>
    "spmd.yield"() : () -> ()
  }) {operandSegmentSizes = array<i32: 1, 1, 1>} : (index, index, index) -> ()
  func.return
}
