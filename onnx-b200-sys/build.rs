// Links libonnxb200.so, the C-ABI library of this repository (CUDA for sm_100a,
// built by nvcc through onnx-rs_b200/csrc/Makefile).  When the library is not
// there yet and ONNXB200_LIB_DIR does not point elsewhere, the Makefile is run.
use std::path::PathBuf;
use std::process::Command;

fn main() {
    println!("cargo:rerun-if-env-changed=ONNXB200_LIB_DIR");
    let manifest = PathBuf::from(std::env::var("CARGO_MANIFEST_DIR").expect("CARGO_MANIFEST_DIR"));
    let pkg = manifest.join("..").join("onnx-rs_b200");
    let dir = match std::env::var("ONNXB200_LIB_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => {
            let so = pkg.join("libonnxb200.so");
            if !so.exists() {
                let status = Command::new("make")
                    .arg("-C")
                    .arg(pkg.join("csrc"))
                    .arg("-j8")
                    .status()
                    .expect("running make for libonnxb200.so (needs nvcc)");
                assert!(status.success(), "make -C onnx-rs_b200/csrc failed");
            }
            println!("cargo:rerun-if-changed={}", so.display());
            pkg.clone()
        }
    };
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=onnxb200");
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
    println!("cargo:include={}", manifest.join("..").join("include").display());
}
