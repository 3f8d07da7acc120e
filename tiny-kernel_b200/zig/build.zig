//! Builds the Zig kernel API against libtkcuda (make -C tiny-kernel_b200 first): the reference's
//! build.zig with the Metal / Foundation / CoreGraphics frameworks (its lines 13-16) replaced by
//! the static CUDA library, the static CUDA runtime, the driver and libstdc++.  Not built
//! here: there is no Zig toolchain on the build or GPU machines.
const std = @import("std");

pub fn build(b: *std.Build) void {
    const target = b.standardTargetOptions(.{});
    const optimize = b.standardOptimizeOption(.{});
    const mod = b.createModule(.{
        .root_source_file = b.path("src/main.zig"),
        .target = target,
        .optimize = optimize,
    });
    mod.addIncludePath(b.path("../../include"));
    mod.addObjectFile(b.path("../lib/libtkcuda.a"));
    mod.linkSystemLibrary("cudart_static", .{});
    mod.linkSystemLibrary("cuda", .{});
    mod.linkSystemLibrary("dl", .{});
    mod.linkSystemLibrary("rt", .{});
    mod.linkSystemLibrary("pthread", .{});
    mod.linkSystemLibrary("stdc++", .{});
    mod.linkSystemLibrary("c", .{});
    const lib = b.addLibrary(.{ .linkage = .static, .name = "tiny-kernel-cuda", .root_module = mod });
    b.installArtifact(lib);
}
