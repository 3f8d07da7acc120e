//! Library root for the CUDA build of the kernel API (the reference's src/main.zig exports with
//! the Metal runtime replaced by src/cuda/cuda.zig).  Not built here (no Zig toolchain on the
//! build or GPU machines).
pub const cuda = @import("cuda/cuda.zig");
pub const quantized = @import("kernels/quantized.zig");
pub const fused = @import("kernels/fused.zig");
pub const rmsnorm = @import("kernels/rmsnorm.zig");

pub const Device = cuda.Device;
pub const Buffer = cuda.Buffer;

/// tk.init() (reference src/main.zig:17-19)
pub fn init() !*Device {
    return Device.init();
}

/// tk.deinit() (reference src/main.zig:21-23)
pub fn deinit(device: *Device) void {
    device.deinit();
}
