// Links libmxmoe.so (built by burn-extended_b200/build.py) and the CUDA
// runtime it shares with its host process.
//   MXMOE_LIB_DIR  directory of libmxmoe.so (default: the in-tree build)
//   CUDA_HOME      CUDA toolkit (default /usr/local/cuda)
use std::env;
use std::path::PathBuf;

fn main() {
    let manifest = PathBuf::from(env::var("CARGO_MANIFEST_DIR").unwrap());
    let default_lib = manifest.join("../../burn-extended_b200/mxmoe");
    let lib_dir = env::var("MXMOE_LIB_DIR").map(PathBuf::from).unwrap_or(default_lib);
    let cuda = env::var("CUDA_HOME").unwrap_or_else(|_| "/usr/local/cuda".to_string());
    println!("cargo:rustc-link-search=native={}", lib_dir.display());
    println!("cargo:rustc-link-search=native={}/lib64", cuda);
    println!("cargo:rustc-link-lib=dylib=mxmoe");
    println!("cargo:rustc-link-lib=dylib=cudart");
    // the library is loaded from its build directory at run time
    println!("cargo:rustc-link-arg=-Wl,-rpath,{}", lib_dir.display());
    println!("cargo:rerun-if-env-changed=MXMOE_LIB_DIR");
    println!("cargo:rerun-if-env-changed=CUDA_HOME");
}
