// swift-tools-version: 5.9
// The Linux drop-in for the reference engine's Metal layer (reference Package.swift:1-12): the C
// module over include/plamo.h and Swift classes `Runtime` and `Batch` with the reference's member
// names, backed by libplamo_cuda.so. The engine's executable target depends on "PlamoCUDA" in place
// of its Metal sources (Runtime.swift, Batch.swift, Packed.swift, Kernels.metal, Batch.metal).
// Build the library first (python plamo3-0.8b-runtime_b200/build.py); the -L flag below points at
// plamo3-0.8b-runtime_b200/lib, where that build puts libplamo_cuda.so. No Swift toolchain exists
// on the build machine of this repository, so this package is checked only as far as its C module:
// the module's shim header compiles as C (tests/test_abi_c_caller.py).
import PackageDescription

let package = Package(
    name: "PlamoCUDA",
    products: [.library(name: "PlamoCUDA", targets: ["PlamoCUDA"])],
    targets: [
        .systemLibrary(name: "CPlamo", path: "Sources/CPlamo"),
        .target(name: "PlamoCUDA", dependencies: ["CPlamo"], path: "Sources/PlamoCUDA",
                linkerSettings: [.unsafeFlags(["-L../lib", "-Xlinker", "-rpath", "-Xlinker", "$ORIGIN/../lib"])]),
    ]
)
