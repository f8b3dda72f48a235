// build.rs for the candle-moe crate linked against the prebuilt Blackwell library.
//
// Replaces the reference crate's build.rs (build.rs:1-103), which compiles kernels/*.cu with
// bindgen_cuda into a static libmoe.a.  Here nothing is compiled: the kernels are prebuilt for
// sm_100a into libcandle_moe_b200.so (python candle-moe_b200/build.py), which exports the same
// two C symbols the crate's src/ffi.rs declares, plus the extended entry points of
// include/candle_moe.h.  The CUDA runtime is linked statically into that library, so no
// cudart/stdc++ link lines are needed.
//
// Not compiled in the image this library was built in (no cargo there): unverified.
use std::path::PathBuf;

fn main() {
    println!("cargo:rerun-if-changed=build.rs");
    println!("cargo:rerun-if-env-changed=CANDLE_MOE_B200_DIR");
    let dir = match std::env::var("CANDLE_MOE_B200_DIR") {
        Ok(d) => PathBuf::from(d),
        Err(_) => panic!(
            "set CANDLE_MOE_B200_DIR to the directory that holds libcandle_moe_b200.so \
             (built by `python candle-moe_b200/build.py`)"
        ),
    };
    let lib = dir.join("libcandle_moe_b200.so");
    if !lib.exists() {
        panic!("{} does not exist", lib.display());
    }
    println!("cargo:rustc-link-search=native={}", dir.display());
    println!("cargo:rustc-link-lib=dylib=candle_moe_b200");
    // find the library at run time without LD_LIBRARY_PATH
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", dir.display());
}
