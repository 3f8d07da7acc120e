//! QMatMulInt4 over libtkcuda: the reference's kernel API (src/kernels/quantized.zig:6-51) with
//! the Metal dispatch replaced by tk_qmatmul_int4.  Same buffers, same layout (w_packed [K/2][N],
//! f16 scales [K/group][N], zero points [K/group][N/2]), same synchronous forward().  Differences
//! the header documents: all m rows are computed (the shader computes row 0) and k is not capped
//! at 4096.  Not built here (no Zig toolchain on the build or GPU machines).
const cuda = @import("../cuda/cuda.zig");
const c = cuda.c;

pub const QMatMulInt4 = struct {
    device: *cuda.Device,

    pub fn init(device: *cuda.Device) !QMatMulInt4 {
        return .{ .device = device };
    }

    pub fn forward(
        self: *QMatMulInt4,
        x: *cuda.Buffer(f32),
        w_packed: *cuda.Buffer(u8),
        scales: *cuda.Buffer(f16),
        zeros: *cuda.Buffer(u8),
        out: *cuda.Buffer(f32),
        m: u32,
        k: u32,
        n: u32,
        group_size: u32,
    ) !void {
        try cuda.check(c.tk_qmatmul_int4(self.device.ctx, x.handle, w_packed.handle,
            @ptrCast(scales.handle), zeros.handle, out.handle, m, k, n, group_size));
    }
};

/// One INT4 matrix (w_packed, scales, zeros) as the FFN entry points take it.
pub const Int4Weights = struct {
    w_packed: *cuda.Buffer(u8),
    scales: *cuda.Buffer(f16),
    zeros: *cuda.Buffer(u8),

    pub fn raw(self: Int4Weights) c.tk_int4_matrix {
        return .{
            .w_packed = self.w_packed.handle,
            .scales = @ptrCast(self.scales.handle),
            .zeros = self.zeros.handle,
        };
    }
};
