//! RMSNorm over libtkcuda (reference src/kernels/rmsnorm.zig:6-43): out = x * rsqrt(mean(x^2) + eps)
//! * weight per row of `dim`; rows = x.count / dim as the reference derives them.  Not built
//! here (no Zig toolchain on the build or GPU machines).
const cuda = @import("../cuda/cuda.zig");
const c = cuda.c;

pub const RMSNorm = struct {
    device: *cuda.Device,

    pub fn init(device: *cuda.Device) !RMSNorm {
        return .{ .device = device };
    }

    pub fn forward(
        self: *RMSNorm,
        x: *cuda.Buffer(f32),
        weight: *cuda.Buffer(f32),
        out: *cuda.Buffer(f32),
        dim: u32,
        eps: f32,
    ) !void {
        const rows: u32 = @intCast(x.count / dim);
        try cuda.check(c.tk_rmsnorm(self.device.ctx, x.handle, weight.handle, out.handle, rows, dim, eps));
    }
};
