//! Fused kernels over libtkcuda: the reference's FusedRMSNormRoPE, Matvec, MatvecDual and
//! FusedSiluMul (src/kernels/fused.zig:6-134, 178-213) with the same forward() arguments, plus
//! the additive INT4 FFN (rmsnorm -> gate/up -> silu(gate)*up -> down [+ x], the reference's
//! bench composition src/bench.zig:266-341 with the down projection of src/model/llama.zig:220-231)
//! and its tensor-parallel form.  Every forward() is synchronous like the reference's.  Not built
//! here (no Zig toolchain on the build or GPU machines).
const cuda = @import("../cuda/cuda.zig");
const quantized = @import("quantized.zig");
const c = cuda.c;

pub const FusedRMSNormRoPE = struct {
    device: *cuda.Device,

    pub fn init(device: *cuda.Device) !FusedRMSNormRoPE {
        return .{ .device = device };
    }

    pub fn forward(
        self: *FusedRMSNormRoPE,
        x: *cuda.Buffer(f32),
        weight: *cuda.Buffer(f32),
        cos_cache: *cuda.Buffer(f32),
        sin_cache: *cuda.Buffer(f32),
        out: *cuda.Buffer(f32),
        dim: u32,
        head_dim: u32,
        pos: u32,
        eps: f32,
    ) !void {
        const rows: u32 = @intCast(x.count / dim);
        try cuda.check(c.tk_fused_rmsnorm_rope(self.device.ctx, x.handle, weight.handle,
            cos_cache.handle, sin_cache.handle, out.handle, rows, dim, head_dim, pos, eps));
    }
};

pub const Matvec = struct {
    device: *cuda.Device,

    pub fn init(device: *cuda.Device) !Matvec {
        return .{ .device = device };
    }

    /// out[n] = sum_k W[n*K + k] * x[k]
    pub fn forward(self: *Matvec, x: *cuda.Buffer(f32), W: *cuda.Buffer(f32), out: *cuda.Buffer(f32),
        K: u32, N: u32) !void {
        try cuda.check(c.tk_matvec(self.device.ctx, x.handle, W.handle, out.handle, K, N));
    }
};

pub const MatvecDual = struct {
    device: *cuda.Device,

    pub fn init(device: *cuda.Device) !MatvecDual {
        return .{ .device = device };
    }

    pub fn forward(self: *MatvecDual, x: *cuda.Buffer(f32), W1: *cuda.Buffer(f32),
        W2: *cuda.Buffer(f32), out1: *cuda.Buffer(f32), out2: *cuda.Buffer(f32), K: u32, N: u32) !void {
        try cuda.check(c.tk_matvec_dual(self.device.ctx, x.handle, W1.handle, W2.handle, out1.handle,
            out2.handle, K, N));
    }
};

pub const FusedSiluMul = struct {
    device: *cuda.Device,

    pub fn init(device: *cuda.Device) !FusedSiluMul {
        return .{ .device = device };
    }

    /// out = silu(gate) * up over gate.count elements
    pub fn forward(self: *FusedSiluMul, gate: *cuda.Buffer(f32), up: *cuda.Buffer(f32),
        out: *cuda.Buffer(f32)) !void {
        const n: u32 = @intCast(gate.count);
        try cuda.check(c.tk_silu_mul(self.device.ctx, gate.handle, up.handle, out.handle, n));
    }
};

/// The INT4 Llama FFN in one call (no counterpart struct in the reference).
pub const FusedInt4FFN = struct {
    device: *cuda.Device,

    pub fn init(device: *cuda.Device) !FusedInt4FFN {
        return .{ .device = device };
    }

    /// out = down(silu(gate(rmsnorm(x))) * up(rmsnorm(x))) (+ x when residual); h receives the
    /// f32 intermediate when given.
    pub fn forward(
        self: *FusedInt4FFN,
        x: *cuda.Buffer(f32),
        norm_weight: *cuda.Buffer(f32),
        gate: quantized.Int4Weights,
        up: quantized.Int4Weights,
        down: quantized.Int4Weights,
        out: *cuda.Buffer(f32),
        h: ?*cuda.Buffer(f32),
        m: u32,
        hidden: u32,
        inter: u32,
        group_size: u32,
        eps: f32,
        residual: bool,
    ) !void {
        const g = gate.raw();
        const u = up.raw();
        const d = down.raw();
        try cuda.check(c.tk_int4_ffn(self.device.ctx, x.handle, norm_weight.handle, &g, &u, &d,
            out.handle, if (h) |b| b.handle else null, m, hidden, inter, group_size, eps,
            if (residual) c.TK_FFN_RESIDUAL else 0));
    }

    /// forward() with x and out in pinned host memory (Device.createHostBuffer): at 1-2 rows the
    /// kernel reads x and writes out over the host link itself, and repeated calls with the same
    /// arguments replay one recorded CUDA graph (TK_FFN_HOST_IO).
    pub fn forwardHostIo(
        self: *FusedInt4FFN,
        x: *cuda.Buffer(f32),
        norm_weight: *cuda.Buffer(f32),
        gate: quantized.Int4Weights,
        up: quantized.Int4Weights,
        down: quantized.Int4Weights,
        out: *cuda.Buffer(f32),
        m: u32,
        hidden: u32,
        inter: u32,
        group_size: u32,
        eps: f32,
        residual: bool,
    ) !void {
        const g = gate.raw();
        const u = up.raw();
        const d = down.raw();
        try cuda.check(c.tk_int4_ffn(self.device.ctx, x.handle, norm_weight.handle, &g, &u, &d,
            out.handle, null, m, hidden, inter, group_size, eps,
            c.TK_FFN_HOST_IO | (if (residual) c.TK_FFN_RESIDUAL else 0)));
    }
};

/// Tensor-parallel INT4 FFN: rank r of `nranks` holds the gate/up columns and down rows
/// [r*I/tp, (r+1)*I/tp); forward() computes the shard and sums the partial outputs over the group
/// (NVLink peer memory or NCCL inside libtkcuda).  Every rank makes the same calls in the same
/// order.
pub const Int4FFNGroup = struct {
    group: *c.tk_tp,

    /// Rank 0 makes the id (newId) and hands it to the others over any channel.
    pub fn newId() ![c.TK_TP_UNIQUE_ID_BYTES]u8 {
        var id: [c.TK_TP_UNIQUE_ID_BYTES]u8 = undefined;
        try cuda.check(c.tk_tp_unique_id(&id));
        return id;
    }

    pub fn init(device: *cuda.Device, nranks: c_int, rank: c_int, id: *const [c.TK_TP_UNIQUE_ID_BYTES]u8) !Int4FFNGroup {
        var g: ?*c.tk_tp = null;
        try cuda.check(c.tk_tp_create(device.ctx, nranks, rank, id, &g));
        return .{ .group = g.? };
    }

    pub fn deinit(self: *Int4FFNGroup) void {
        c.tk_tp_destroy(self.group);
    }

    pub fn forward(
        self: *Int4FFNGroup,
        x: *cuda.Buffer(f32),
        norm_weight: *cuda.Buffer(f32),
        gate: quantized.Int4Weights,
        up: quantized.Int4Weights,
        down: quantized.Int4Weights,
        out: *cuda.Buffer(f32),
        m: u32,
        hidden: u32,
        inter_shard: u32,
        group_size: u32,
        eps: f32,
        residual: bool,
    ) !void {
        const g = gate.raw();
        const u = up.raw();
        const d = down.raw();
        try cuda.check(c.tk_int4_ffn_tp(self.group, x.handle, norm_weight.handle, &g, &u, &d,
            out.handle, m, hidden, inter_shard, group_size, eps,
            if (residual) c.TK_FFN_RESIDUAL else 0));
    }
};
