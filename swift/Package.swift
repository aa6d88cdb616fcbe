// swift-tools-version: 5.9
// SwiftPM binding of the CUDA sampling engine (libtgsample.so, include/tgsample.h).
// CTGSample is the C shim module over the C ABI; TGSample is the Swift wrapper a
// serve loop calls in place of its MLX sampling (Serve.swift:1483-1506) and
// speculative verification (SpeculativeDecode.swift:41-210).
//
// Build (Linux, with the library built in-tree):
//   swift build -Xlinker -L../tinygpt_b200 -Xlinker -rpath -Xlinker ../tinygpt_b200
import PackageDescription

let package = Package(
    name: "TGSample",
    products: [
        .library(name: "TGSample", targets: ["TGSample"]),
    ],
    targets: [
        .target(
            name: "CTGSample",
            path: "Sources/CTGSample",
            publicHeadersPath: "include",
            linkerSettings: [.linkedLibrary("tgsample")]
        ),
        .target(name: "TGSample", dependencies: ["CTGSample"], path: "Sources/TGSample"),
    ]
)
