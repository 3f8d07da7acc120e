//! Runtime layer over libtkcuda (include/tk_cuda.h) for the reference's Zig kernel API.
//!
//! Takes the place of the Metal runtime (src/metal/metal.zig, device.zig, buffer.zig, objc.zig
//! of Lulzx/tiny-kernel): a Device owns one CUDA device context of the library (its stream and
//! the scratch its kernels use), Buffer(T) is caller-owned memory with a `handle` and a `count`
//! like the Metal buffer, and every kernel struct calls one `tk_*` entry point.
//! Not built here: there is no Zig toolchain on the build or GPU machines; the same C symbols
//! are exercised through Python ctypes by the repository's tests.
const std = @import("std");
pub const c = @cImport(@cInclude("tk_cuda.h"));

pub const Error = error{
    InvalidArgument,
    CudaFailure,
    NcclFailure,
    DeviceWaitTimedOut,
    Unsupported,
    OutOfMemory,
};

/// Maps a tk_* status to a Zig error (the reference's forward() can fail only on command buffer
/// or encoder creation; here argument checks and device-side timeouts report too).
pub fn check(status: c_int) Error!void {
    switch (status) {
        c.TK_OK => return,
        c.TK_ERR_ARG => return error.InvalidArgument,
        c.TK_ERR_CUDA => return error.CudaFailure,
        c.TK_ERR_NCCL => return error.NcclFailure,
        c.TK_ERR_TIMEOUT => return error.DeviceWaitTimedOut,
        c.TK_ERR_UNSUPPORTED => return error.Unsupported,
        else => return error.OutOfMemory,
    }
}

/// The text of the last failure on this thread (tk_last_error_string).
pub fn lastError() []const u8 {
    return std.mem.span(c.tk_last_error_string());
}

pub const Device = struct {
    ctx: *c.tk_device,
    allocator: std.mem.Allocator,

    /// Device.init (reference src/metal/device.zig:10-12): CUDA device 0.
    pub fn init() !*Device {
        return initWithAllocator(std.heap.page_allocator);
    }

    pub fn initWithAllocator(allocator: std.mem.Allocator) !*Device {
        return initOrdinal(allocator, 0);
    }

    /// One Device per GPU: the tensor-parallel FFN runs one process (or thread) per ordinal.
    pub fn initOrdinal(allocator: std.mem.Allocator, ordinal: c_int) !*Device {
        var ctx: ?*c.tk_device = null;
        try check(c.tk_device_create(ordinal, &ctx));
        const self = try allocator.create(Device);
        self.* = .{ .ctx = ctx.?, .allocator = allocator };
        return self;
    }

    pub fn deinit(self: *Device) void {
        c.tk_device_destroy(self.ctx);
        self.allocator.destroy(self);
    }

    pub fn name(self: *Device) []const u8 {
        return std.mem.span(c.tk_device_name(self.ctx));
    }

    /// Host-visible (managed) memory, the counterpart of MTLResourceStorageModeShared.
    pub fn createBuffer(self: *Device, comptime T: type, count: usize) !Buffer(T) {
        return Buffer(T).init(self, count);
    }

    /// Pinned host memory (TK_MEM_HOST): the x / out of FusedInt4FFN.forwardHostIo.
    pub fn createHostBuffer(self: *Device, comptime T: type, count: usize) !Buffer(T) {
        return Buffer(T).initKind(self, count, c.TK_MEM_HOST);
    }

    pub fn createBufferWithData(self: *Device, comptime T: type, data: []const T) !Buffer(T) {
        var b = try Buffer(T).init(self, data.len);
        @memcpy(b.slice(), data);
        return b;
    }

    /// Waits for everything queued on the device's stream (the reference waits per command
    /// buffer: CommandBuffer.waitUntilCompleted).
    pub fn synchronize(self: *Device) !void {
        try check(c.tk_device_synchronize(self.ctx));
    }
};

pub fn Buffer(comptime T: type) type {
    return struct {
        /// Device address of the first element (managed memory: also valid on the host).
        handle: [*]T,
        count: usize,
        device: *Device,

        const Self = @This();

        pub fn init(device: *Device, count: usize) !Self {
            return initKind(device, count, c.TK_MEM_SHARED);
        }

        /// kind: TK_MEM_SHARED (managed), TK_MEM_HOST (pinned host) or TK_MEM_DEVICE.
        pub fn initKind(device: *Device, count: usize, kind: c_int) !Self {
            var p: ?*anyopaque = null;
            try check(c.tk_buffer_alloc(device.ctx, count * @sizeOf(T), kind, &p));
            return .{ .handle = @ptrCast(@alignCast(p.?)), .count = count, .device = device };
        }

        pub fn deinit(self: *Self) void {
            _ = c.tk_buffer_free(self.device.ctx, self.handle);
        }

        /// Host view; waits for the device's queued work first (every forward() is synchronous,
        /// so after a forward the view already holds its results).
        pub fn slice(self: *Self) []T {
            _ = c.tk_device_synchronize(self.device.ctx);
            return self.handle[0..self.count];
        }

        pub fn constSlice(self: *const Self) []const T {
            _ = c.tk_device_synchronize(self.device.ctx);
            return self.handle[0..self.count];
        }
    };
}
