// Swift drop-ins for the quantized modules of Qwen38Core, over libq38's C ABI (CQ38).
//
// They replace, at the same call sites, the MLX modules the reference builds:
//   QuantizedLinear            Sources/Qwen38Core/FlashNext/Qwen4ExpPrequantized.swift:77-106, call :156-159
//   Qwen38HadamardQuantizedLinear  Sources/Qwen38Core/Bonsai2/Qwen38HadamardModules.swift:24-40
//   QuantizedSwitchLinear      Vendor/mlx-swift-lm-local.patch:184-218 (gatherQuantizedMM)
//   SwitchGLU + router         Sources/Qwen38Core/FlashNext/Qwen4ExpSparseMoE.swift:208-214, 275-294
//   Qwen4ExpPrequantizedEmbedding  Sources/Qwen38Core/FlashNext/Qwen4ExpPrequantized.swift:108-160
// Parameter names (weight, scales, biases) and shapes are the checkpoint's, so a loader
// fills them from the same safetensors keys.  Tensors are device buffers owned by the
// caller (Q38Tensor); every call is enqueued on the context's stream.
//
// This file is not compiled in the build container (no Swift toolchain there); it is
// written against include/q38.h, which the C tests exercise.
import CQ38

public struct Q38Failure: Error, CustomStringConvertible {
    public let status: q38_status
    public let message: String
    public var description: String { "q38 \(status.rawValue): \(message)" }
}

/// A device buffer with its logical shape and element type.  The pointer is a device
/// address (cudaMalloc'd by the host application); nothing here owns or frees it.
public struct Q38Tensor {
    public var pointer: UnsafeMutableRawPointer
    public var shape: [Int]
    public var dtype: q38_dtype
    public init(pointer: UnsafeMutableRawPointer, shape: [Int], dtype: q38_dtype) {
        self.pointer = pointer
        self.shape = shape
        self.dtype = dtype
    }
    public var rows: Int64 { Int64(shape.dropLast().reduce(1, *)) }
    public var lastDim: Int64 { Int64(shape.last ?? 0) }
    var u32: UnsafePointer<UInt32> { UnsafePointer(pointer.assumingMemoryBound(to: UInt32.self)) }
    var i32: UnsafeMutablePointer<Int32> { pointer.assumingMemoryBound(to: Int32.self) }
}

/// One libq38 context: a device, a stream and the library's workspace.  One per host
/// thread and device, as the library requires.
public final class Q38Context {
    public let handle: OpaquePointer
    public init(device: Int32, stream: UnsafeMutableRawPointer? = nil) throws {
        var h: OpaquePointer?
        let st = q38_ctx_create(device, &h)
        guard st == Q38_OK, let h else { throw Q38Failure(status: st, message: "context on device \(device)") }
        handle = h
        if let stream { q38_ctx_set_stream(handle, stream) }
    }
    deinit { q38_ctx_destroy(handle) }

    public func check(_ st: q38_status) throws {
        guard st == Q38_OK else {
            throw Q38Failure(status: st, message: String(cString: q38_last_error(handle)))
        }
    }
    /// Synchronises the stream and reports device-side timeouts and out-of-range indices.
    public func checkDevice() throws { try check(q38_ctx_check_device(handle)) }
}

/// QuantizedLinear.callAsFunction: y = quantizedMM(x, weight, scales, biases, transpose: true).
public final class Q38QuantizedLinear {
    public let weight: Q38Tensor, scales: Q38Tensor, biases: Q38Tensor?
    public let groupSize: Int32, bits: Int32
    public init(weight: Q38Tensor, scales: Q38Tensor, biases: Q38Tensor?, groupSize: Int, bits: Int) {
        self.weight = weight; self.scales = scales; self.biases = biases
        self.groupSize = Int32(groupSize); self.bits = Int32(bits)
    }
    public var outputDimensions: Int64 { Int64(weight.shape[0]) }

    public func callAsFunction(_ ctx: Q38Context, _ x: Q38Tensor, into y: Q38Tensor) throws {
        try ctx.check(q38_quantized_matmul(ctx.handle, x.pointer, x.rows, x.lastDim, x.dtype, weight.u32,
                                           scales.pointer, biases?.pointer, scales.dtype, outputDimensions,
                                           1, groupSize, bits, Q38_MODE_AFFINE, y.pointer))
    }
}

/// Qwen38HadamardQuantizedLinear: rotate x (signs, block), round to x's dtype, then the product.
public final class Q38HadamardQuantizedLinear {
    public let linear: Q38QuantizedLinear
    public let signs: UnsafePointer<Float>?
    public let block: Int32
    public init(linear: Q38QuantizedLinear, signs: UnsafePointer<Float>?, block: Int) {
        self.linear = linear; self.signs = signs; self.block = Int32(block)
    }
    public func callAsFunction(_ ctx: Q38Context, _ x: Q38Tensor, into y: Q38Tensor) throws {
        let l = linear
        try ctx.check(q38_hadamard_quantized_matmul(ctx.handle, x.pointer, x.rows, x.lastDim, x.dtype, signs, block,
                                                    l.weight.u32, l.scales.pointer, l.biases?.pointer, l.scales.dtype,
                                                    l.outputDimensions, l.groupSize, l.bits, y.pointer))
    }
}

/// The gated MLP down(silu(gate(x)) * up(x)); gate and up share one pass over both weights.
public final class Q38QuantizedMLP {
    public let gate: Q38QuantizedLinear, up: Q38QuantizedLinear, down: Q38QuantizedLinear
    public init(gate: Q38QuantizedLinear, up: Q38QuantizedLinear, down: Q38QuantizedLinear) {
        self.gate = gate; self.up = up; self.down = down
    }
    /// `h` is scratch of shape [M, intermediate] in x's dtype.
    public func callAsFunction(_ ctx: Q38Context, _ x: Q38Tensor, hidden h: Q38Tensor, into y: Q38Tensor) throws {
        try ctx.check(q38_quantized_gate_up(ctx.handle, x.pointer, x.rows, x.lastDim, x.dtype,
                                            gate.weight.u32, gate.scales.pointer, gate.biases?.pointer,
                                            up.weight.u32, up.scales.pointer, up.biases?.pointer, gate.scales.dtype,
                                            gate.outputDimensions, gate.groupSize, gate.bits, Q38_MODE_AFFINE,
                                            h.pointer))
        try down(ctx, h, into: y)
    }
}

/// QuantizedSwitchLinear.callAsFunction(x, indices): gatherQuantizedMM over expert stacks
/// weight [E, N, K*bits/32], scales/biases [E, N, K/group].
public final class Q38QuantizedSwitchLinear {
    public let weight: Q38Tensor, scales: Q38Tensor, biases: Q38Tensor?
    public let groupSize: Int32, bits: Int32
    public init(weight: Q38Tensor, scales: Q38Tensor, biases: Q38Tensor?, groupSize: Int, bits: Int) {
        self.weight = weight; self.scales = scales; self.biases = biases
        self.groupSize = Int32(groupSize); self.bits = Int32(bits)
    }
    /// x [Bx, M, K]; rhs (expert of each output) int32 [P]; lhs (row of x) int32 [P] or nil.
    public func callAsFunction(_ ctx: Q38Context, _ x: Q38Tensor, lhs: Q38Tensor?, rhs: Q38Tensor,
                               sortedIndices: Bool, into out: Q38Tensor) throws {
        let E = Int64(weight.shape[0]), N = Int64(weight.shape[1])
        let Bx = Int64(x.shape[0]), M = Int64(x.shape.count > 2 ? x.shape[1] : 1)
        try ctx.check(q38_gather_quantized_matmul(ctx.handle, x.pointer, Bx, M, x.lastDim, x.dtype, weight.u32,
                                                  scales.pointer, biases?.pointer, scales.dtype, E, N,
                                                  lhs.map { UnsafePointer($0.i32) }, UnsafePointer(rhs.i32),
                                                  Int64(rhs.shape.reduce(1, *)), 1, groupSize, bits, Q38_MODE_AFFINE,
                                                  sortedIndices ? 1 : 0, out.pointer))
    }
}

/// Routed experts of Qwen4ExpSparseMoE: router (gate Linear, softmax, top-k, renormalise)
/// then SwitchGLU with the weighted expert sum.
public final class Q38SparseMoE {
    public let router: Q38Tensor  // bf16 [E, H]
    public let gate: Q38QuantizedSwitchLinear, up: Q38QuantizedSwitchLinear, down: Q38QuantizedSwitchLinear
    public let topK: Int32, normalizeTopK: Bool
    /// Qwen4ExpSharedExpert and shared_expert_gate ([1, H]); nil for a block without them.
    public let sharedExpert: Q38QuantizedMLP?, sharedExpertGate: Q38QuantizedLinear?
    public init(router: Q38Tensor, gate: Q38QuantizedSwitchLinear, up: Q38QuantizedSwitchLinear,
                down: Q38QuantizedSwitchLinear, topK: Int, normalizeTopK: Bool,
                sharedExpert: Q38QuantizedMLP? = nil, sharedExpertGate: Q38QuantizedLinear? = nil) {
        self.router = router; self.gate = gate; self.up = up; self.down = down
        self.topK = Int32(topK); self.normalizeTopK = normalizeTopK
        self.sharedExpert = sharedExpert; self.sharedExpertGate = sharedExpertGate
    }
    /// indices int32 [T, topK] and scores bf16 [T, topK] are scratch the caller provides.
    public func callAsFunction(_ ctx: Q38Context, _ x: Q38Tensor, indices: Q38Tensor, scores: Q38Tensor,
                               into out: Q38Tensor) throws {
        let T = x.rows, H = x.lastDim, E = Int64(router.shape[0]), I = Int64(gate.weight.shape[1])
        try ctx.check(q38_moe_route(ctx.handle, x.pointer, T, H, x.dtype, router.pointer, E, topK,
                                    normalizeTopK ? 1 : 0, indices.i32, scores.pointer, nil))
        try ctx.check(q38_switch_glu(ctx.handle, x.pointer, T, H, I, E, topK, UnsafePointer(indices.i32),
                                     scores.pointer, gate.weight.u32, gate.scales.pointer, gate.biases?.pointer,
                                     up.weight.u32, up.scales.pointer, up.biases?.pointer,
                                     down.weight.u32, down.scales.pointer, down.biases?.pointer,
                                     Q38_BF16, gate.groupSize, gate.bits, out.pointer))
        // + sigmoid(shared_expert_gate(x)) * sharedExpert(x), in place (Qwen4ExpSparseMoE.swift:295-298)
        if let se = sharedExpert, let sg = sharedExpertGate {
            try ctx.check(q38_shared_expert(ctx.handle, x.pointer, T, H, se.gate.outputDimensions,
                                            se.gate.weight.u32, se.gate.scales.pointer, se.gate.biases?.pointer,
                                            se.up.weight.u32, se.up.scales.pointer, se.up.biases?.pointer,
                                            se.down.weight.u32, se.down.scales.pointer, se.down.biases?.pointer,
                                            sg.weight.u32, sg.scales.pointer, sg.biases?.pointer,
                                            se.gate.scales.dtype, se.gate.groupSize, se.gate.bits,
                                            out.pointer, out.pointer))
        }
    }
}

/// Qwen4ExpPrequantizedEmbedding: lookup (callAsFunction) and the tied projection (asLinear).
public final class Q38QuantizedEmbedding {
    public let table: Q38QuantizedLinear
    public init(weight: Q38Tensor, scales: Q38Tensor, biases: Q38Tensor?, groupSize: Int, bits: Int) {
        table = Q38QuantizedLinear(weight: weight, scales: scales, biases: biases, groupSize: groupSize, bits: bits)
    }
    public func callAsFunction(_ ctx: Q38Context, ids: Q38Tensor, into out: Q38Tensor) throws {
        let t = table
        let dims = Int64(t.weight.shape[1]) * 32 / Int64(t.bits)
        try ctx.check(q38_quantized_embedding(ctx.handle, UnsafePointer(ids.i32), Int64(ids.shape.reduce(1, *)),
                                              t.weight.u32, t.scales.pointer, t.biases?.pointer, t.scales.dtype,
                                              t.outputDimensions, dims, t.groupSize, t.bits, Q38_MODE_AFFINE,
                                              out.pointer, out.dtype))
    }
    public func asLinear(_ ctx: Q38Context, _ x: Q38Tensor, into y: Q38Tensor) throws {
        try table(ctx, x, into: y)
    }
}

// ------------------------------------------------------------------ several GPUs

/// One NCCL rank of libq38 (NCCL is loaded by the library).  Rank 0 creates the id with
/// `Q38Communicator.uniqueID()` and hands its bytes to the other ranks over any channel.
public final class Q38Communicator {
    public let handle: OpaquePointer
    public let rank: Int32, world: Int32
    public static func uniqueID() throws -> q38_comm_id {
        var id = q38_comm_id()
        let st = q38_comm_get_unique_id(&id)
        guard st == Q38_OK else { throw Q38Failure(status: st, message: String(cString: q38_comm_error())) }
        return id
    }
    public init(id: q38_comm_id, world: Int32, rank: Int32, device: Int32, timeoutMs: Int32 = 60_000) throws {
        var id = id
        var h: OpaquePointer?
        let st = q38_comm_init_rank(&id, world, rank, device, timeoutMs, &h)
        guard st == Q38_OK, let h else { throw Q38Failure(status: st, message: String(cString: q38_comm_error())) }
        handle = h
        self.rank = rank
        self.world = world
    }
    deinit { q38_comm_destroy(handle) }
    /// After a peer failed: abort the collectives in flight.
    public func abort() { q38_comm_abort(handle) }
}

/// The dense MLP with gate/up split by output rows and down by its reduction dimension;
/// `callAsFunction` leaves the all-reduced y on every rank.
public final class Q38TensorParallelMLP {
    public let gate: Q38QuantizedLinear, up: Q38QuantizedLinear, down: Q38QuantizedLinear
    public let chunks: Int32
    public init(gate: Q38QuantizedLinear, up: Q38QuantizedLinear, down: Q38QuantizedLinear, chunks: Int = 4) {
        self.gate = gate; self.up = up; self.down = down; self.chunks = Int32(chunks)
    }
    public func callAsFunction(_ ctx: Q38Context, _ comm: Q38Communicator, _ x: Q38Tensor, into y: Q38Tensor) throws {
        try ctx.check(q38_tp_mlp(ctx.handle, comm.handle, x.pointer, x.rows, x.lastDim,
                                 gate.weight.u32, gate.scales.pointer, gate.biases?.pointer,
                                 up.weight.u32, up.scales.pointer, up.biases?.pointer,
                                 down.weight.u32, down.scales.pointer, down.biases?.pointer,
                                 gate.outputDimensions, Q38_BF16, gate.groupSize, gate.bits, chunks, y.pointer))
    }
}

/// SwitchGLU with this rank's share of the experts; every rank uses the same capacity.
public final class Q38ExpertParallelSwitchGLU {
    public let gate: Q38QuantizedSwitchLinear, up: Q38QuantizedSwitchLinear, down: Q38QuantizedSwitchLinear
    public let numExperts: Int64, capacity: Int64
    public init(gate: Q38QuantizedSwitchLinear, up: Q38QuantizedSwitchLinear, down: Q38QuantizedSwitchLinear,
                numExperts: Int, capacity: Int) {
        self.gate = gate; self.up = up; self.down = down
        self.numExperts = Int64(numExperts); self.capacity = Int64(capacity)
    }
    public func callAsFunction(_ ctx: Q38Context, _ comm: Q38Communicator, _ x: Q38Tensor, indices: Q38Tensor,
                               scores: Q38Tensor, into out: Q38Tensor) throws {
        let I = Int64(gate.weight.shape[1]), k = Int32(indices.lastDim)
        try ctx.check(q38_ep_switch_glu(ctx.handle, comm.handle, x.pointer, x.rows, x.lastDim, I, numExperts, k,
                                        UnsafePointer(indices.i32), scores.pointer,
                                        gate.weight.u32, gate.scales.pointer, gate.biases?.pointer,
                                        up.weight.u32, up.scales.pointer, up.biases?.pointer,
                                        down.weight.u32, down.scales.pointer, down.biases?.pointer,
                                        Q38_BF16, gate.groupSize, gate.bits, capacity, out.pointer))
    }
}
